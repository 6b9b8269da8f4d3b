// Q-prep in exact arithmetic (MLA_PREC_EXACT): steps 2a1, 2a-norm, 2a2, 2b and
// 2c of the absorbed MLA forward on CUDA cores, for fp32 / fp64 / fp16 / bf16
// storage. Reference semantics: launch_q_absorbed (mla_kernels.cu:599-767) and
// the PyTorch path prepare_q_mla_absorbed (exhaustive_benchmark_suite.py:268-286).
//
//   2a1  P1[z] = x[:, kz] @ W_q_a[kz, :]            split-K partials (acc dtype)
//   2an  q_lat = T( sum_z P1[z] * rsqrt(mean(.^2)+eps) * gain )
//   2a2  P2[z] = q_lat[:, kz] @ W_q_b[kz, :]        split-K partials (acc dtype)
//   2b   q_nope = sum_z P2[z][.., nope cols], q_rope = T(RoPE(sum_z P2[z][.., rope cols]))
//   2c   q_absorbed[:, h] = T(q_nope[:, h] @ W_uk[h])
//
// Split-K partials are reduced by the next kernel, never with atomics, so the
// result is deterministic run to run.
#include "qprep.cuh"
#include "simt_gemm.cuh"
#include "tc_gemm.cuh"

#include <cmath>
#include <type_traits>

namespace mla {
namespace {

// C[z][m][n] = sum_{k in slice z} A[m][k] * B[k][n]; A and B row-major.
template <typename TA, typename TB, typename Acc>
struct ProjProblem {
    static constexpr bool kAKFast = true;
    static constexpr bool kBNFast = true;
    const TA* A; const TB* B;
    int64_t lda, ldb, M, N, m0, n0;
    __device__ Acc a(int64_t ml, int64_t k) const {
        const int64_t m = m0 + ml;
        return (m < M) ? cvt<Acc>(A[m * lda + k]) : Acc(0);
    }
    __device__ Acc b(int64_t k, int64_t nl) const {
        const int64_t n = n0 + nl;
        return (n < N) ? cvt<Acc>(B[k * ldb + n]) : Acc(0);
    }
};

// One launch of a split-K projection. grid = (n tiles, m tiles, splits).
template <class Cfg, typename TA, typename TB>
__global__ void __launch_bounds__(256) proj_splitk_kernel(
    const TA* __restrict__ A, const TB* __restrict__ B, typename Cfg::Acc* __restrict__ C,
    int64_t M, int64_t N, int64_t K, int64_t k_chunk)
{
    using Acc = typename Cfg::Acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ProjProblem<TA, TB, Acc> p{A, B, K, N, M, N,
                               int64_t(blockIdx.y) * Cfg::BM, int64_t(blockIdx.x) * Cfg::BN};
    const int64_t kb = int64_t(blockIdx.z) * k_chunk;
    const int64_t ke = (kb + k_chunk < K) ? kb + k_chunk : K;
    Acc acc[Cfg::TM][Cfg::TN];
    simt_gemm_mainloop<Cfg>(p, kb, ke, acc, reinterpret_cast<Acc*>(smem_raw));
    const int tx = threadIdx.x % Cfg::kTX, ty = threadIdx.x / Cfg::kTX;
    Acc* Cz = C + int64_t(blockIdx.z) * M * N;
#pragma unroll
    for (int i = 0; i < Cfg::TM; ++i) {
        const int64_t m = p.m0 + Cfg::m_of(ty, i);
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < Cfg::TN; ++j) {
            const int64_t n = p.n0 + Cfg::n_of(tx, j);
            if (n < N) Cz[m * N + n] = acc[i][j];
        }
    }
}

// 2a-norm: one block per row. Sums the split-K partials, RMS-normalises with
// the gain and narrows to the storage dtype (the reference hands the latent to
// 2a2 in the input dtype: mla_kernels.cu:416-419).
template <typename T>
__global__ void __launch_bounds__(256) lat_norm_kernel(
    const acc_t<T>* __restrict__ P1, int splits, const T* __restrict__ gain,
    T* __restrict__ q_lat, int64_t M, int64_t q_lora, acc_t<T> eps)
{
    using Acc = acc_t<T>;
    constexpr int kKeep = 8;            // values kept in registers per thread (q_lora <= 2048)
    const int64_t m = blockIdx.x;
    auto val = [&](int64_t n) {
        Acc v = Acc(0);
        for (int z = 0; z < splits; ++z) v += P1[(int64_t(z) * M + m) * q_lora + n];
        return v;
    };
    const bool keep = q_lora <= int64_t(kKeep) * blockDim.x;
    Acc kept[kKeep];
    Acc ss = Acc(0);
    if (keep) {   // one pass over the partials
#pragma unroll
        for (int e = 0; e < kKeep; ++e) {
            const int64_t n = threadIdx.x + int64_t(e) * blockDim.x;
            kept[e] = (n < q_lora) ? val(n) : Acc(0);
            ss = fma(kept[e], kept[e], ss);
        }
    } else {
        for (int64_t n = threadIdx.x; n < q_lora; n += blockDim.x) {
            const Acc v = val(n);
            ss = fma(v, v, ss);
        }
    }
    __shared__ Acc red[32];
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        Acc t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : Acc(0);
        for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
        if (threadIdx.x == 0) red[0] = Acc(1) / sqrt(t / Acc(q_lora) + eps);
    }
    __syncthreads();
    const Acc inv_rms = red[0];
    if (keep) {
#pragma unroll
        for (int e = 0; e < kKeep; ++e) {
            const int64_t n = threadIdx.x + int64_t(e) * blockDim.x;
            if (n < q_lora) q_lat[m * q_lora + n] = cvt<T>(kept[e] * inv_rms * cvt<Acc>(gain[n]));
        }
    } else {
        for (int64_t n = threadIdx.x; n < q_lora; n += blockDim.x)
            q_lat[m * q_lora + n] = cvt<T>(val(n) * inv_rms * cvt<Acc>(gain[n]));
    }
}

// 2b: reduce the 2a2 partials of every head into q_nope (acc dtype, the left
// operand of 2c) and rotate the rope slice. Interleaved pairs (2j, 2j+1) are
// rotated by pos * inv_freq[j], inv_freq[j] = 1 / 10000^(2j/rope), the
// convention of apply_rope (exhaustive_benchmark_suite.py:210-232).
template <typename T>
struct RopeTable { acc_t<T> inv_freq[kMaxRopePairs]; };

// cos / sin of every (query index, pair): cs[s][j] = {cos, sin}(pos[s] * inv_freq[j]),
// narrowed to the storage dtype as apply_rope does (exhaustive_benchmark_suite.py:222-223).
template <typename T>
__global__ void __launch_bounds__(256) rope_table_kernel(const int64_t* __restrict__ positions, int64_t sq,
                                                         int64_t pairs, RopeTable<T> tab, acc_t<T>* __restrict__ cs)
{
    using Acc = acc_t<T>;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < sq * pairs;
         i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t s = i / pairs, j = i % pairs;
        const Acc ang = Acc(positions[s]) * tab.inv_freq[j];
        cs[2 * i] = cvt<Acc>(cvt<T>(cos(ang)));
        cs[2 * i + 1] = cvt<Acc>(cvt<T>(sin(ang)));
    }
}

template <typename T, typename NopeT = acc_t<T>>
__global__ void __launch_bounds__(256) rope_gather_kernel(
    const acc_t<T>* __restrict__ P2, int splits, const int64_t* __restrict__ positions,
    NopeT* __restrict__ q_nope, T* __restrict__ q_rope,
    int64_t M, int64_t sq, int64_t heads, int64_t nope, int64_t rope, const acc_t<T>* __restrict__ cs)
{
    using Acc = acc_t<T>;
    const int64_t qk = nope + rope;
    const int64_t ncols = heads * qk;
    const int64_t per_head = nope + rope / 2;
    const int64_t total = M * heads * per_head;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int64_t e = idx % per_head;
        const int64_t mh = idx / per_head;
        const int64_t h = mh % heads;
        const int64_t m = mh / heads;
        const int64_t col = h * qk + (e < nope ? e : nope + 2 * (e - nope));
        auto sum = [&](int64_t c) {
            Acc v = Acc(0);
            for (int z = 0; z < splits; ++z) v += P2[(int64_t(z) * M + m) * ncols + c];
            return v;
        };
        if (e < nope) {
            q_nope[mh * nope + e] = cvt<NopeT>(sum(col));
        } else {
            const int64_t j = e - nope;
            const Acc ev = sum(col), od = sum(col + 1);
            const Acc* t = cs + 2 * ((m % sq) * (rope / 2) + j);
            const Acc c = t[0], s = t[1];
            q_rope[mh * rope + 2 * j] = cvt<T>(ev * c - od * s);
            q_rope[mh * rope + 2 * j + 1] = cvt<T>(ev * s + od * c);
        }
    }
}

// Vectorised 2a-norm for an fp32 accumulator: one block of 256 threads per row,
// each thread owning up to kVec float4 pieces of the row, all split-K partial loads
// of a piece issued together. Same sums, in the same order, as lat_norm_kernel.
template <typename T, typename OutT = T>
__global__ void __launch_bounds__(1024) lat_norm_vec_kernel(
    const float* __restrict__ P1, int splits, const T* __restrict__ gain,
    OutT* __restrict__ q_lat, int64_t M, int64_t q_lora, float eps)
{
    pdl_wait();
    pdl_trigger();
    constexpr int kMaxSplits = 16;                 // all split loads of a piece in flight at once
    const int64_t m = blockIdx.x;
    const int n4 = int(q_lora / 4);
    const int c = threadIdx.x;                     // one float4 piece of the row per thread
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < n4) {
        float4 t[kMaxSplits];
#pragma unroll
        for (int z = 0; z < kMaxSplits; ++z)
            if (z < splits) t[z] = __ldg(reinterpret_cast<const float4*>(P1 + (int64_t(z) * M + m) * q_lora) + c);
#pragma unroll
        for (int z = 0; z < kMaxSplits; ++z)
            if (z < splits) { v.x += t[z].x; v.y += t[z].y; v.z += t[z].z; v.w += t[z].w; }
    }
    float ss = v.x * v.x;
    ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
    __shared__ float red[32];
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) tot += red[w];
    const float inv_rms = 1.f / sqrtf(tot / float(q_lora) + eps);
    if (c < n4) {
        const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            q_lat[m * q_lora + 4 * c + k] = cvt<OutT>(f[k] * inv_rms * cvt<float>(gain[4 * c + k]));
    }
}

template <typename T>
mla_status_t launch_lat_norm(const acc_t<T>* P1, int splits, const T* gain, T* q_lat, int64_t M, int64_t q_lora,
                             double eps, cudaStream_t st) {
    if constexpr (std::is_same<acc_t<T>, float>::value) {
        if (q_lora % 4 == 0 && q_lora <= 4096 && splits <= 16) {
            const unsigned threads = unsigned((q_lora / 4 + 31) / 32 * 32);
            lat_norm_vec_kernel<T><<<unsigned(M), threads, 0, st>>>(P1, splits, gain, q_lat, M, q_lora, float(eps));
            return check_launch("q latent RMSNorm (2a-norm)");
        }
    }
    lat_norm_kernel<T><<<unsigned(M), 256, 0, st>>>(P1, splits, gain, q_lat, M, q_lora, acc_t<T>(eps));
    return check_launch("q latent RMSNorm (2a-norm)");
}

// Vectorised 2b for an fp32 accumulator: one warp per (token, head), float4 loads
// of the split-K partials; same arithmetic as rope_gather_kernel.
template <typename NopeT>
__device__ __forceinline__ void store4(NopeT* dst, float a, float b, float c, float d) {
    if constexpr (std::is_same<NopeT, float>::value) {
        *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
    } else {
        dst[0] = cvt<NopeT>(a); dst[1] = cvt<NopeT>(b); dst[2] = cvt<NopeT>(c); dst[3] = cvt<NopeT>(d);
    }
}

template <typename T, typename NopeT>
__global__ void __launch_bounds__(256) rope_gather_vec_kernel(
    const float* __restrict__ P2, int splits, NopeT* __restrict__ q_nope, T* __restrict__ q_rope,
    int64_t M, int64_t sq, int64_t heads, int64_t nope, int64_t rope, const int64_t* __restrict__ positions,
    const RopeTable<T> tab)
{
    const int lane = threadIdx.x & 31;
    const int64_t qk = nope + rope;
    const int64_t ncols = heads * qk;
    const int64_t rows = M * heads;
    for (int64_t mh = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; mh < rows;
         mh += (int64_t(gridDim.x) * blockDim.x) >> 5) {
        const int64_t m = mh / heads, h = mh - m * heads;
        const float* src = P2 + m * ncols + h * qk;
        const int64_t zstride = M * ncols;
        auto sum4 = [&](int64_t col) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int z = 0; z < splits; ++z) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(src + z * zstride + col));
                v.x += t.x; v.y += t.y; v.z += t.z; v.w += t.w;
            }
            return v;
        };
        for (int64_t c = 4 * lane; c < nope; c += 128) {
            const float4 v = sum4(c);
            store4<NopeT>(q_nope + mh * nope + c, v.x, v.y, v.z, v.w);
        }
        const float pos = float(positions[m % sq]);
        for (int64_t c = 4 * lane; c < rope; c += 128) {
            const float4 v = sum4(nope + c);                   // pairs j = c/2 and c/2 + 1
            const int64_t j = c / 2;
            // cos / sin in the accumulate dtype narrowed to the storage dtype, as
            // rope_table_kernel computes them
            const float a0 = pos * tab.inv_freq[j], a1 = pos * tab.inv_freq[j + 1];
            const float c0 = cvt<float>(cvt<T>(cos(a0))), s0 = cvt<float>(cvt<T>(sin(a0)));
            const float c1 = cvt<float>(cvt<T>(cos(a1))), s1 = cvt<float>(cvt<T>(sin(a1)));
            T* o = q_rope + mh * rope + c;
            o[0] = cvt<T>(v.x * c0 - v.y * s0);
            o[1] = cvt<T>(v.x * s0 + v.y * c0);
            o[2] = cvt<T>(v.z * c1 - v.w * s1);
            o[3] = cvt<T>(v.z * s1 + v.w * c1);
        }
    }
}

// 2b launcher. The vectorised kernel computes its cos / sin inline; the generic
// one reads them from a table (cs, in the workspace) filled first.
template <typename T, typename NopeT>
mla_status_t launch_rope_gather(const acc_t<T>* P2, int splits, const int64_t* positions, NopeT* q_nope, T* q_rope,
                                int64_t M, int64_t sq, int64_t heads, int64_t nope, int64_t rope,
                                const RopeTable<T>& tab, acc_t<T>* cs, cudaStream_t st) {
    if constexpr (std::is_same<acc_t<T>, float>::value) {
        if (nope % 4 == 0 && rope % 4 == 0) {
            int64_t blocks = ceil_div(M * heads, 8);
            if (blocks > 32LL * sm_count()) blocks = 32LL * sm_count();
            rope_gather_vec_kernel<T, NopeT><<<unsigned(blocks), 256, 0, st>>>(P2, splits, q_nope, q_rope, M, sq,
                                                                             heads, nope, rope, positions, tab);
            return check_launch("q rope (2b)");
        }
    }
    const int64_t tblocks = ceil_div(sq * (rope / 2), 256);
    rope_table_kernel<T><<<unsigned(tblocks > 0 ? tblocks : 1), 256, 0, st>>>(positions, sq, rope / 2, tab, cs);
    MLA_TRY(check_launch("q rope table"));
    const int64_t total = M * heads * (nope + rope / 2);
    int64_t blocks = ceil_div(total, 256);
    const int64_t cap = 16LL * sm_count();
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    rope_gather_kernel<T, NopeT><<<unsigned(blocks), 256, 0, st>>>(P2, splits, positions, q_nope, q_rope, M, sq,
                                                                   heads, nope, rope, cs);
    return check_launch("q rope (2b)");
}

// 2c: q_absorbed[m, h, :] = q_nope[m, h, :] @ W_uk[h]. grid = (n tiles, m tiles, heads).
template <typename T, typename Acc>
struct AbsorbProblem {
    static constexpr bool kAKFast = true;
    static constexpr bool kBNFast = true;
    const Acc* qn; const T* W;
    int64_t M, heads, nope, R, h, m0, n0;
    __device__ Acc a(int64_t ml, int64_t k) const {
        const int64_t m = m0 + ml;
        return (m < M) ? qn[(m * heads + h) * nope + k] : Acc(0);
    }
    __device__ Acc b(int64_t k, int64_t nl) const {
        const int64_t n = n0 + nl;
        return (n < R) ? cvt<Acc>(W[(h * nope + k) * R + n]) : Acc(0);
    }
};

template <class Cfg, typename T>
__global__ void __launch_bounds__(256) absorb_kernel(
    const typename Cfg::Acc* __restrict__ q_nope, const T* __restrict__ W_uk,
    T* __restrict__ q_abs, int64_t M, int64_t heads, int64_t nope, int64_t R)
{
    using Acc = typename Cfg::Acc;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    AbsorbProblem<T, Acc> p{q_nope, W_uk, M, heads, nope, R, int64_t(blockIdx.z),
                            int64_t(blockIdx.y) * Cfg::BM, int64_t(blockIdx.x) * Cfg::BN};
    Acc acc[Cfg::TM][Cfg::TN];
    simt_gemm_mainloop<Cfg>(p, 0, nope, acc, reinterpret_cast<Acc*>(smem_raw));
    const int tx = threadIdx.x % Cfg::kTX, ty = threadIdx.x / Cfg::kTX;
#pragma unroll
    for (int i = 0; i < Cfg::TM; ++i) {
        const int64_t m = p.m0 + Cfg::m_of(ty, i);
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < Cfg::TN; ++j) {
            const int64_t n = p.n0 + Cfg::n_of(tx, j);
            if (n < R) q_abs[(m * heads + p.h) * R + n] = cvt<T>(acc[i][j]);
        }
    }
}

struct QPlan {
    bool small;          // 16-row tiles (B*Sq <= 16)
    int64_t bm, bn, bk;
    int split1, split2;
    int64_t chunk1, chunk2;
    size_t off_p1, off_qlat, off_p2, off_qnope, off_cs, total;
};

// Split-K plan: enough CTAs for ~4 resident waves, each split a whole number of
// K tiles, no empty split.
void plan_split(int64_t tiles, int64_t K, int64_t bk, int& split, int64_t& chunk) {
    const int64_t want = 4LL * 2 * sm_count();
    int64_t s = want / (tiles > 0 ? tiles : 1);
    const int64_t ktiles = ceil_div(K, bk);
    if (s > ktiles / 2) s = ktiles / 2;    // keep at least two K tiles per split
    if (s < 1) s = 1;
    const int64_t chunk_tiles = ceil_div(ktiles, s);
    s = ceil_div(ktiles, chunk_tiles);
    split = int(s);
    chunk = chunk_tiles * bk;
}

template <typename T>
QPlan make_plan(const QArgs& a) {
    using Acc = acc_t<T>;
    QPlan p{};
    const int64_t M = a.batch * a.sq;
    p.small = M <= 16;
    p.bm = p.small ? CfgSmall<Acc>::BM : CfgBig<Acc>::BM;
    p.bn = p.small ? CfgSmall<Acc>::BN : CfgBig<Acc>::BN;
    p.bk = p.small ? CfgSmall<Acc>::BK : CfgBig<Acc>::BK;
    const int64_t mt = ceil_div(M, p.bm);
    const int64_t ncols = a.heads * (a.nope + a.rope);
    plan_split(mt * ceil_div(a.q_lora, p.bn), a.hidden, p.bk, p.split1, p.chunk1);
    plan_split(mt * ceil_div(ncols, p.bn), a.q_lora, p.bk, p.split2, p.chunk2);
    size_t off = 0;
    p.off_p1 = off;    off = align_up(off + size_t(p.split1) * M * a.q_lora * sizeof(Acc), 256);
    p.off_qlat = off;  off = align_up(off + size_t(M) * a.q_lora * sizeof(T), 256);
    p.off_p2 = off;    off = align_up(off + size_t(p.split2) * M * ncols * sizeof(Acc), 256);
    p.off_qnope = off; off = align_up(off + size_t(M) * a.heads * a.nope * sizeof(Acc), 256);
    p.off_cs = off;    off = align_up(off + size_t(a.sq) * (a.rope / 2 + 1) * 2 * sizeof(Acc), 256);
    p.total = off;
    return p;
}

template <class Cfg, typename TA, typename TB>
mla_status_t launch_proj(const TA* A, const TB* B, typename Cfg::Acc* C, int64_t M, int64_t N,
                         int64_t K, int split, int64_t chunk, cudaStream_t st) {
    auto kern = proj_splitk_kernel<Cfg, TA, TB>;
    if (Cfg::kSmemBytes > 48 * 1024)
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::kSmemBytes));
    dim3 grid(unsigned(ceil_div(N, Cfg::BN)), unsigned(ceil_div(M, Cfg::BM)), unsigned(split));
    kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, st>>>(A, B, C, M, N, K, chunk);
    return check_launch("q projection");
}

template <class Cfg, typename T>
mla_status_t launch_absorb(const typename Cfg::Acc* qn, const T* W, T* out, const QArgs& a,
                           int64_t M, cudaStream_t st) {
    auto kern = absorb_kernel<Cfg, T>;
    if (Cfg::kSmemBytes > 48 * 1024)
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg::kSmemBytes));
    dim3 grid(unsigned(ceil_div(a.kv_rank, Cfg::BN)), unsigned(ceil_div(M, Cfg::BM)), unsigned(a.heads));
    kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, st>>>(qn, W, out, M, a.heads, a.nope, a.kv_rank);
    return check_launch("q absorb (2c)");
}

}  // namespace

template <typename T> size_t qprep_tensor_workspace(const QArgs& a);
template <typename T> mla_status_t qprep_tensor_impl(const QArgs& a, cudaStream_t st, bool split3);

// The exact path runs the tensor-core pipeline wherever the shapes allow TMA
// tiles: fp32 storage with 3xTF32 GEMMs (fp32-class products, fp32
// accumulation); 16-bit storage with kind::f16 GEMMs, whose 16-bit products are
// exact in fp32 and accumulate in fp32 (the reference's policy for 16-bit
// storage, with the same 16-bit intermediates). fp64 stays on CUDA cores.
template <typename T>
bool exact_uses_tc(const QArgs& a) { return !std::is_same<T, double>::value && qprep_tensor_supported<T>(a); }

template <typename T>
size_t qprep_exact_workspace(const QArgs& a) {
    return exact_uses_tc<T>(a) ? qprep_tensor_workspace<T>(a) : make_plan<T>(a).total;
}

template <typename T>
mla_status_t qprep_exact(const QArgs& a, cudaStream_t st) {
    using Acc = acc_t<T>;
    if (exact_uses_tc<T>(a)) return qprep_tensor_impl<T>(a, st, std::is_same<T, float>::value);
    const QPlan p = make_plan<T>(a);
    const int64_t M = a.batch * a.sq;
    const int64_t ncols = a.heads * (a.nope + a.rope);
    char* ws = static_cast<char*>(a.workspace);
    Acc* P1 = reinterpret_cast<Acc*>(ws + p.off_p1);
    T* q_lat = reinterpret_cast<T*>(ws + p.off_qlat);
    Acc* P2 = reinterpret_cast<Acc*>(ws + p.off_p2);
    Acc* q_nope = reinterpret_cast<Acc*>(ws + p.off_qnope);
    const T* x = static_cast<const T*>(a.x);
    const T* Wqa = static_cast<const T*>(a.W_q_a);
    const T* Wqb = static_cast<const T*>(a.W_q_b);

    if (p.small) {
        MLA_TRY((launch_proj<CfgSmall<Acc>, T, T>(x, Wqa, P1, M, a.q_lora, a.hidden, p.split1, p.chunk1, st)));
    } else {
        MLA_TRY((launch_proj<CfgBig<Acc>, T, T>(x, Wqa, P1, M, a.q_lora, a.hidden, p.split1, p.chunk1, st)));
    }
    MLA_TRY(launch_lat_norm<T>(P1, p.split1, static_cast<const T*>(a.q_norm_w), q_lat, M, a.q_lora, a.eps, st));
    if (p.small) {
        MLA_TRY((launch_proj<CfgSmall<Acc>, T, T>(q_lat, Wqb, P2, M, ncols, a.q_lora, p.split2, p.chunk2, st)));
    } else {
        MLA_TRY((launch_proj<CfgBig<Acc>, T, T>(q_lat, Wqb, P2, M, ncols, a.q_lora, p.split2, p.chunk2, st)));
    }

    RopeTable<T> tab{};
    for (int64_t j = 0; j < a.rope / 2; ++j) {
        // Rounded the way torch computes 1 / 10000 ** (2j / rope) in the
        // accumulate dtype: a correctly rounded power, then an IEEE divide.
        const double pw = std::pow(10000.0, double(2 * j) / double(a.rope));
        tab.inv_freq[j] = Acc(1) / Acc(pw);
    }
    {
        Acc* cs = reinterpret_cast<Acc*>(ws + p.off_cs);
        MLA_TRY((launch_rope_gather<T, Acc>(P2, p.split2, a.positions, q_nope, static_cast<T*>(a.q_rope), M, a.sq,
                                            a.heads, a.nope, a.rope, tab, cs, st)));
    }
    if (p.small) {
        MLA_TRY((launch_absorb<CfgSmall<Acc>, T>(q_nope, static_cast<const T*>(a.W_uk),
                                                 static_cast<T*>(a.q_absorbed), a, M, st)));
    } else {
        MLA_TRY((launch_absorb<CfgBig<Acc>, T>(q_nope, static_cast<const T*>(a.W_uk),
                                               static_cast<T*>(a.q_absorbed), a, M, st)));
    }
    return MLA_OK;
}

template size_t qprep_exact_workspace<float>(const QArgs&);
template size_t qprep_exact_workspace<double>(const QArgs&);
template size_t qprep_exact_workspace<__half>(const QArgs&);
template size_t qprep_exact_workspace<__nv_bfloat16>(const QArgs&);
template mla_status_t qprep_exact<float>(const QArgs&, cudaStream_t);
template mla_status_t qprep_exact<double>(const QArgs&, cudaStream_t);
template mla_status_t qprep_exact<__half>(const QArgs&, cudaStream_t);
template mla_status_t qprep_exact<__nv_bfloat16>(const QArgs&, cudaStream_t);

// ------------------------------------------------------------ tensor-core Q-prep
// MLA_PREC_TENSOR: 2a1 and 2a2 run as split-K tcgen05 GEMMs (kind::tf32 for
// fp32 storage, kind::f16 for 16-bit) writing fp32 partials that the same
// RMSNorm and RoPE kernels reduce; 2c is a per-head tcgen05 GEMM whose left
// operand, q_nope, is rounded to the storage dtype.
namespace {

struct QTPlan {
    int split1, split2;
    int64_t chunk1, chunk2;
    size_t off_p1, off_qlat, off_p2, off_qnope, off_cs, total;
};

// Split-K plan of a weight-streaming GEMM (one CTA per SM): the slice count s
// minimises (rounds of CTAs * SMs / units) + s * 2M/K, the time of the weight
// stream relative to a perfectly balanced one plus the fp32 partials each slice
// writes and the next kernel reads (M*N per slice against K*N weights); at
// least four K blocks per slice.
int tc_split(int64_t tiles, int64_t M, int64_t K, int64_t bk, int64_t& chunk) {
    const int64_t kblocks = ceil_div(K, bk);
    const int64_t sms = sm_count();
    int64_t best = 1;
    double best_cost = 1e30;
    for (int64_t s = 1; s <= 32 && s <= (kblocks / 4 > 1 ? kblocks / 4 : 1); ++s) {
        const int64_t cb = ceil_div(kblocks, s);
        const int64_t slices = ceil_div(kblocks, cb);            // non-empty slices
        const int64_t units = tiles * slices;
        const double cost = double(ceil_div(units, sms) * sms) / double(units) + double(slices) * 2.0 * double(M) / double(K);
        if (cost < best_cost - 1e-9) { best_cost = cost; best = s; }
    }
    const int64_t cb = ceil_div(kblocks, best);
    chunk = cb * bk;
    return int(ceil_div(kblocks, cb));
}

template <typename T>
QTPlan make_tplan(const QArgs& a) {
    using Acc = acc_t<T>;
    QTPlan p{};
    const int64_t M = a.batch * a.sq;
    const int64_t ncols = a.heads * (a.nope + a.rope);
    const int64_t bk = tc_gemm_bk<T>();
    const int64_t mt = ceil_div(M, 128);
    p.split1 = tc_split(mt * ceil_div(a.q_lora, 128), M, a.hidden, bk, p.chunk1);
    p.split2 = tc_split(mt * ceil_div(ncols, 128), M, a.q_lora, bk, p.chunk2);
    size_t off = 0;
    p.off_p1 = off;    off = align_up(off + size_t(p.split1) * M * a.q_lora * sizeof(Acc), 256);
    p.off_qlat = off;  off = align_up(off + size_t(M) * a.q_lora * sizeof(T), 256);
    p.off_p2 = off;    off = align_up(off + size_t(p.split2) * M * ncols * sizeof(Acc), 256);
    p.off_qnope = off; off = align_up(off + size_t(M) * a.heads * a.nope * sizeof(Acc), 256);
    p.off_cs = off;    off = align_up(off + size_t(a.sq) * (a.rope / 2 + 1) * 2 * sizeof(Acc), 256);
    p.total = off;
    return p;
}

}  // namespace

template <typename T>
bool qprep_tensor_supported(const QArgs& a) {
    if constexpr (std::is_same<T, double>::value) return false;
    else {
        constexpr int64_t v = 16 / sizeof(T);   // TMA: 16-byte strides
        const int64_t ncols = a.heads * (a.nope + a.rope);
        return a.q_lora % 32 == 0 && ncols % 32 == 0 && a.kv_rank % 32 == 0 && a.hidden % v == 0 &&
               a.q_lora % v == 0 && a.nope % v == 0 && a.batch * a.sq > 0;
    }
}

template <typename T>
size_t qprep_tensor_workspace(const QArgs& a) { return make_tplan<T>(a).total; }

template <typename T>
mla_status_t qprep_tensor(const QArgs& a, cudaStream_t st) { return qprep_tensor_impl<T>(a, st, false); }

template <typename T>
mla_status_t qprep_tensor_impl(const QArgs& a, cudaStream_t st, bool split3) {
    using Acc = acc_t<T>;
    const QTPlan p = make_tplan<T>(a);
    const int64_t M = a.batch * a.sq;
    const int64_t ncols = a.heads * (a.nope + a.rope);
    char* ws = static_cast<char*>(a.workspace);
    DeviceStatus* dst = nullptr;
    MLA_TRY(device_status_block(&dst));
    int* err = &dst->code;
    Acc* P1 = reinterpret_cast<Acc*>(ws + p.off_p1);
    T* q_lat = reinterpret_cast<T*>(ws + p.off_qlat);
    Acc* P2 = reinterpret_cast<Acc*>(ws + p.off_p2);
    T* q_nope_t = reinterpret_cast<T*>(ws + p.off_qnope);
    TcGemm g1{};   // 2a1: x [M, hidden] @ W_q_a [hidden, q_lora]
    g1.A = a.x; g1.a_dims[0] = a.hidden; g1.a_dims[1] = 1; g1.a_dims[2] = M; g1.a_ld[0] = a.hidden; g1.a_ld[1] = a.hidden;
    g1.B = a.W_q_a; g1.b_mn = true; g1.b_dims[0] = a.q_lora; g1.b_dims[1] = a.hidden; g1.b_dims[2] = 1;
    g1.b_ld[0] = a.q_lora; g1.b_ld[1] = a.q_lora * a.hidden;
    g1.M = M; g1.N = a.q_lora; g1.K = a.hidden; g1.Z = p.split1; g1.spb = p.split1; g1.k_chunk = p.chunk1;
    g1.C = P1; g1.c_is_t = false; g1.c_ldm = a.q_lora; g1.c_ldz = M * a.q_lora; g1.bn = 128; g1.err = err; g1.split3 = split3;
    MLA_TRY(tc_gemm<T>(g1, st));

    MLA_TRY(launch_lat_norm<T>(P1, p.split1, static_cast<const T*>(a.q_norm_w), q_lat, M, a.q_lora, a.eps, st));

    TcGemm g2{};   // 2a2: q_lat [M, q_lora] @ W_q_b [q_lora, H*(nope+rope)]
    g2.A = q_lat; g2.a_dims[0] = a.q_lora; g2.a_dims[1] = 1; g2.a_dims[2] = M; g2.a_ld[0] = a.q_lora; g2.a_ld[1] = a.q_lora;
    g2.B = a.W_q_b; g2.b_mn = true; g2.b_dims[0] = ncols; g2.b_dims[1] = a.q_lora; g2.b_dims[2] = 1;
    g2.b_ld[0] = ncols; g2.b_ld[1] = ncols * a.q_lora;
    g2.M = M; g2.N = ncols; g2.K = a.q_lora; g2.Z = p.split2; g2.spb = p.split2; g2.k_chunk = p.chunk2;
    g2.C = P2; g2.c_is_t = false; g2.c_ldm = ncols; g2.c_ldz = M * ncols; g2.bn = 128; g2.err = err; g2.split3 = split3;
    MLA_TRY(tc_gemm<T>(g2, st));

    RopeTable<T> tab{};
    for (int64_t j = 0; j < a.rope / 2; ++j) {
        const double pw = std::pow(10000.0, double(2 * j) / double(a.rope));
        tab.inv_freq[j] = Acc(1) / Acc(pw);
    }
    {
        // q_nope in the storage dtype: the left operand of the 2c tensor-core GEMM,
        // whose operands share one dtype
        Acc* cs = reinterpret_cast<Acc*>(ws + p.off_cs);
        MLA_TRY((launch_rope_gather<T, T>(P2, p.split2, a.positions, q_nope_t, static_cast<T*>(a.q_rope), M, a.sq,
                                          a.heads, a.nope, a.rope, tab, cs, st)));
    }
    TcGemm g3{};   // 2c: per head, q_nope[:, h, :] @ W_uk[h]
    g3.A = q_nope_t; g3.a_dims[0] = a.nope; g3.a_dims[1] = a.heads; g3.a_dims[2] = M;
    g3.a_ld[0] = a.nope; g3.a_ld[1] = a.heads * a.nope;
    g3.B = a.W_uk; g3.b_mn = true; g3.b_dims[0] = a.kv_rank; g3.b_dims[1] = a.nope; g3.b_dims[2] = a.heads;
    g3.b_ld[0] = a.kv_rank; g3.b_ld[1] = a.nope * a.kv_rank;
    g3.M = M; g3.N = a.kv_rank; g3.K = a.nope; g3.Z = int(a.heads); g3.spb = 1; g3.k_chunk = a.nope;
    g3.C = a.q_absorbed; g3.c_is_t = true; g3.c_ldm = a.heads * a.kv_rank; g3.c_ldz = a.kv_rank;
    g3.bn = a.kv_rank % 256 == 0 ? 256 : 128; g3.err = err; g3.split3 = split3;
    return tc_gemm<T>(g3, st);
}

// ------------------------------------------------------- pre-packed weights
// fp32 storage, MLA_PREC_TENSOR: the three Q-prep weights are converted once to
// bf16 (mla_pack_q_weights) and the projections run as kind::f16 tcgen05 GEMMs
// on them, so each call streams half the weight bytes of the kind::tf32 path.
// x is cast to bf16 per call (its 128 x 7168 values are small next to the
// weights); split-K partials, the RMSNorm and the RoPE stay fp32; q_lat and
// q_nope, the left operands of 2a2 and 2c, are bf16; q_absorbed and q_rope are
// written in fp32.
namespace {

__global__ void __launch_bounds__(256) cast_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                                        int64_t n4) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src) + i);
        __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t*>(&lo);
        o.y = *reinterpret_cast<uint32_t*>(&hi);
        reinterpret_cast<uint2*>(dst)[i] = o;
    }
}

mla_status_t cast_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t st) {
    const int64_t n4 = n / 4;
    int64_t blocks = ceil_div(n4, 256);
    if (blocks > 8LL * sm_count()) blocks = 8LL * sm_count();
    if (blocks < 1) blocks = 1;
    launch_pdl(cast_bf16_kernel, dim3(unsigned(blocks)), dim3(256), 0, st, src, dst, n4);
    return check_launch("bf16 cast");
}

struct PackLayout {
    size_t off_qa, off_qb, off_uk, total;
};

PackLayout pack_layout(int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank) {
    PackLayout l{};
    size_t off = 0;
    l.off_qa = off; off = align_up(off + size_t(hidden) * q_lora * 2, 256);
    l.off_qb = off; off = align_up(off + size_t(q_lora) * heads * (nope + rope) * 2, 256);
    l.off_uk = off; off = align_up(off + size_t(heads) * nope * kv_rank * 2, 256);
    l.total = off;
    return l;
}

struct QPPlan {
    int split1, split2;
    int64_t chunk1, chunk2;
    size_t off_x, off_p1, off_qlat, off_p2, off_qnope, total;
};

QPPlan make_pplan(const QArgs& a) {
    using B16 = __nv_bfloat16;
    QPPlan p{};
    const int64_t M = a.batch * a.sq;
    const int64_t ncols = a.heads * (a.nope + a.rope);
    const int64_t bk = tc_gemm_bk<B16>();
    const int64_t mt = ceil_div(M, 128);
    p.split1 = tc_split(mt * ceil_div(a.q_lora, 128), M, a.hidden, bk, p.chunk1);
    // 2a2 is not split over K: its epilogue splits q per head and applies the RoPE
    p.split2 = 1;
    p.chunk2 = a.q_lora;
    (void)ncols;
    size_t off = 0;
    p.off_x = off;     off = align_up(off + size_t(M) * a.hidden * sizeof(B16), 256);
    p.off_p1 = off;    off = align_up(off + size_t(p.split1) * M * a.q_lora * sizeof(float), 256);
    p.off_qlat = off;  off = align_up(off + size_t(M) * a.q_lora * sizeof(B16), 256);
    p.off_p2 = off;
    p.off_qnope = off; off = align_up(off + size_t(M) * a.heads * a.nope * sizeof(B16), 256);
    p.total = off;
    return p;
}

}  // namespace

mla_status_t cast_to_bf16(const float* src, __nv_bfloat16* dst, int64_t n, cudaStream_t st) {
    return cast_bf16(src, dst, n, st);
}

bool qprep_packed_supported(const QArgs& a) {
    const int64_t ncols = a.heads * (a.nope + a.rope);
    return a.q_lora % 32 == 0 && ncols % 32 == 0 && a.kv_rank % 32 == 0 && a.hidden % 8 == 0 && a.q_lora % 8 == 0 &&
           a.nope % 32 == 0 && a.rope % 32 == 0 && a.rope <= 128 && a.q_lora <= 4096 && a.batch * a.sq > 0 &&
           (a.batch * a.sq * a.hidden) % 4 == 0;
}

size_t pack_q_weights_bytes(int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank) {
    return pack_layout(hidden, q_lora, heads, nope, rope, kv_rank).total;
}

mla_status_t pack_q_weights(const float* W_q_a, const float* W_q_b, const float* W_uk, int64_t hidden, int64_t q_lora,
                            int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank, void* packed,
                            cudaStream_t st) {
    const PackLayout l = pack_layout(hidden, q_lora, heads, nope, rope, kv_rank);
    char* base = static_cast<char*>(packed);
    MLA_TRY(cast_bf16(W_q_a, reinterpret_cast<__nv_bfloat16*>(base + l.off_qa), hidden * q_lora, st));
    MLA_TRY(cast_bf16(W_q_b, reinterpret_cast<__nv_bfloat16*>(base + l.off_qb), q_lora * heads * (nope + rope), st));
    return cast_bf16(W_uk, reinterpret_cast<__nv_bfloat16*>(base + l.off_uk), heads * nope * kv_rank, st);
}

size_t qprep_packed_workspace(const QArgs& a) { return make_pplan(a).total; }

mla_status_t qprep_packed(const QArgs& a, const void* packed, cudaStream_t st) {
    using B16 = __nv_bfloat16;
    const QPPlan p = make_pplan(a);
    const PackLayout l = pack_layout(a.hidden, a.q_lora, a.heads, a.nope, a.rope, a.kv_rank);
    const char* pk = static_cast<const char*>(packed);
    const int64_t M = a.batch * a.sq;
    const int64_t ncols = a.heads * (a.nope + a.rope);
    char* ws = static_cast<char*>(a.workspace);
    DeviceStatus* dst = nullptr;
    MLA_TRY(device_status_block(&dst));
    int* err = &dst->code;
    B16* x16 = reinterpret_cast<B16*>(ws + p.off_x);
    float* P1 = reinterpret_cast<float*>(ws + p.off_p1);
    B16* q_lat = reinterpret_cast<B16*>(ws + p.off_qlat);
    B16* q_nope = reinterpret_cast<B16*>(ws + p.off_qnope);
    MLA_TRY(cast_bf16(static_cast<const float*>(a.x), x16, M * a.hidden, st));

    TcGemm g1{};   // 2a1: x [M, hidden] @ W_q_a [hidden, q_lora], bf16 operands, fp32 partials
    g1.A = x16; g1.a_dims[0] = a.hidden; g1.a_dims[1] = 1; g1.a_dims[2] = M; g1.a_ld[0] = a.hidden; g1.a_ld[1] = a.hidden;
    g1.B = pk + l.off_qa; g1.b_mn = true; g1.b_dims[0] = a.q_lora; g1.b_dims[1] = a.hidden; g1.b_dims[2] = 1;
    g1.b_ld[0] = a.q_lora; g1.b_ld[1] = a.q_lora * a.hidden;
    g1.M = M; g1.N = a.q_lora; g1.K = a.hidden; g1.Z = p.split1; g1.spb = p.split1; g1.k_chunk = p.chunk1;
    g1.C = P1; g1.c_is_t = false; g1.c_ldm = a.q_lora; g1.c_ldz = M * a.q_lora; g1.bn = 128; g1.err = err;
    MLA_TRY(tc_gemm<B16>(g1, st));

    {   // 2a-norm: fp32 arithmetic, bf16 latent for 2a2
        const unsigned threads = unsigned((a.q_lora / 4 + 31) / 32 * 32);
        if (p.split1 > 16) return set_error(MLA_ERR_UNSUPPORTED, "MLA: packed Q-prep split-K above 16");
        launch_pdl(lat_norm_vec_kernel<float, B16>, dim3(unsigned(M)), dim3(threads), 0, st,
                   static_cast<const float*>(P1), int(p.split1), static_cast<const float*>(a.q_norm_w), q_lat, M,
                   int64_t(a.q_lora), float(a.eps));
        MLA_TRY(check_launch("q latent RMSNorm (2a-norm)"));
    }

    // 2a2: q_lat [M, q_lora] @ W_q_b [q_lora, H*(nope+rope)]; the epilogue stores
    // q_nope (bf16) and the rotated q_rope (fp32) directly
    GemmRopeEpilogue re{};
    re.q_nope = q_nope;
    re.q_rope = static_cast<float*>(a.q_rope);
    re.positions = a.positions;
    re.sq = a.sq; re.heads = a.heads; re.nope = a.nope; re.rope = a.rope;
    for (int64_t j = 0; j < a.rope / 2; ++j)   // 1 / fp32(10000^(2j/rope)) in fp32, as apply_rope
        re.inv_freq[j] = 1.0f / float(std::pow(10000.0, double(2 * j) / double(a.rope)));
    TcGemm g2{};
    g2.A = q_lat; g2.a_dims[0] = a.q_lora; g2.a_dims[1] = 1; g2.a_dims[2] = M; g2.a_ld[0] = a.q_lora; g2.a_ld[1] = a.q_lora;
    g2.B = pk + l.off_qb; g2.b_mn = true; g2.b_dims[0] = ncols; g2.b_dims[1] = a.q_lora; g2.b_dims[2] = 1;
    g2.b_ld[0] = ncols; g2.b_ld[1] = ncols * a.q_lora;
    g2.M = M; g2.N = ncols; g2.K = a.q_lora; g2.Z = 1; g2.spb = 1; g2.k_chunk = a.q_lora;
    g2.C = nullptr; g2.c_is_t = false; g2.c_ldm = ncols; g2.c_ldz = M * ncols; g2.err = err;
    // tile width: the fewest waves x columns per tile over the persistent grid (at
    // N = 128 heads x 192 and 148 SMs, 192-column tiles fill one wave with a head each)
    g2.bn = 128;
    int64_t best = INT64_MAX;
    for (const int bn : {128, 192, 256}) {
        const int64_t tiles = ceil_div(ncols, int64_t(bn)) * ceil_div(M, int64_t(128));
        const int64_t cost = ceil_div(tiles, int64_t(sm_count())) * bn;
        if (cost < best) { best = cost; g2.bn = bn; }
    }
    g2.rope_epi = &re;
    MLA_TRY(tc_gemm<B16>(g2, st));

    TcGemm g3{};   // 2c: per head, q_nope[:, h, :] @ W_uk[h], fp32 output
    g3.A = q_nope; g3.a_dims[0] = a.nope; g3.a_dims[1] = a.heads; g3.a_dims[2] = M;
    g3.a_ld[0] = a.nope; g3.a_ld[1] = a.heads * a.nope;
    g3.B = pk + l.off_uk; g3.b_mn = true; g3.b_dims[0] = a.kv_rank; g3.b_dims[1] = a.nope; g3.b_dims[2] = a.heads;
    g3.b_ld[0] = a.kv_rank; g3.b_ld[1] = a.nope * a.kv_rank;
    g3.M = M; g3.N = a.kv_rank; g3.K = a.nope; g3.Z = int(a.heads); g3.spb = 1; g3.k_chunk = a.nope;
    g3.C = a.q_absorbed; g3.c_is_t = false; g3.c_ldm = a.heads * a.kv_rank; g3.c_ldz = a.kv_rank;
    g3.bn = a.kv_rank % 256 == 0 ? 256 : 128; g3.err = err;
    return tc_gemm<B16>(g3, st);
}

#define MLA_QT(T) \
    template bool qprep_tensor_supported<T>(const QArgs&); \
    template size_t qprep_tensor_workspace<T>(const QArgs&); \
    template mla_status_t qprep_tensor<T>(const QArgs&, cudaStream_t); \
    template mla_status_t qprep_tensor_impl<T>(const QArgs&, cudaStream_t, bool);
MLA_QT(float)
MLA_QT(double)
MLA_QT(__half)
MLA_QT(__nv_bfloat16)
#undef MLA_QT

}  // namespace mla
