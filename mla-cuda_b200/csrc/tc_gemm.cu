// Tensor-core GEMM (tcgen05 + TMA) for the dense stages of the MLA forward.
//
// One CTA computes a 128 x BN output tile of one slice / batch z: warp 0 issues
// TMA loads of 128B-swizzled A and B blocks into a ring of stages, warp 1 (one
// thread) issues the MMAs (M = 128, N = BN, K = 8 tf32 or 16 bf16/fp16 per
// instruction) into a TMEM accumulator, warps 2-5 read the accumulator back
// (one TMEM lane = one output row per thread) and store it. The weights of
// these stages are streamed exactly once per 128-row block of activations, so
// at decode batch sizes the kernel is bound by HBM bandwidth on the weights.
//
// fp32 operands run as kind::tf32 (10-bit mantissa, fp32 accumulation); this is
// used only by the tensor-core precision of the MLA entry points.
#include "tc_gemm.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cstdio>
#include <cstdlib>

namespace mla {
namespace tcg {

using namespace sm100;

constexpr int kThreads = 192;
enum : int { ERR_TIMEOUT_BASE = 200 };

struct Run {
    int64_t M, N, K, k_chunk;
    int Z, split, b_mn, c_is_t;
    void* C; int64_t c_ldm, c_ldz;
    int* err;
    int dbg;
};

template <typename T> constexpr uint32_t fmt() {
    return std::is_same<T, float>::value ? 2u : std::is_same<T, __half>::value ? 0u : 1u;
}

// BN = 128 keeps 3 stages (97 KB) so that two CTAs share an SM: a 192-CTA launch
// then runs in one wave on 148 SMs instead of 1.3.
template <int BN> constexpr int stages() { return BN == 256 ? 4 : 3; }
template <typename T, int BN> constexpr int a_bytes() { return 128 * 128; }        // 128 rows x 128 B
template <typename T, int BN> constexpr int b_bytes() { return BN * 128; }         // BN x BK elements
template <typename T, int BN> constexpr size_t smem_bytes() {
    return 1024 + size_t(stages<BN>()) * (a_bytes<T, BN>() + b_bytes<T, BN>()) + 256;
}

template <typename T, int BN>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(
    const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Run r)
{
    constexpr int S = stages<BN>();
    constexpr int BK = tc_gemm_bk<T>();             // elements per 128-byte row
    constexpr int kInstK = 32 / int(sizeof(T));      // K per MMA instruction (32 bytes)
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* As = smem;
    unsigned char* Bs = smem + S * a_bytes<T, BN>();
    uint64_t* full = reinterpret_cast<uint64_t*>(Bs + S * b_bytes<T, BN>());
    uint64_t* empty = full + S;
    uint64_t* acc_full = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    volatile int* abort = abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n0 = int64_t(blockIdx.x) * BN;
    const int64_t m0 = int64_t(blockIdx.y) * 128;
    const int z = blockIdx.z;
    int64_t kb = 0, ke = r.K;
    if (r.split) {
        kb = int64_t(z) * r.k_chunk;
        ke = min(r.K, kb + r.k_chunk);
    }
    const int64_t nkb = ke > kb ? (ke - kb + BK - 1) / BK : 0;
    const int ya = r.split ? 0 : z;      // batch coordinate of A and B

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        for (int64_t i = 0; i < nkb; ++i) {
            const int s = int(i % S);
            if (!mbar_wait(&empty[s], uint32_t(((i / S) & 1) ^ 1), abort, r.err, ERR_TIMEOUT_BASE + 1)) break;
            const int32_t k = int32_t(kb + i * BK);
            mbar_arrive_expect_tx(&full[s], uint32_t(a_bytes<T, BN>() + b_bytes<T, BN>()));
            tma_load_3d(As + s * a_bytes<T, BN>(), &tmA, &full[s], k, ya, int32_t(m0));
            unsigned char* bdst = Bs + s * b_bytes<T, BN>();
            if (r.b_mn) {
                for (int g = 0; g < BN / BK; ++g)   // BK-wide column groups of N, BK rows of K each
                    tma_load_3d(bdst + g * (BK * 128), &tmB, &full[s], int32_t(n0 + g * BK), k, ya);
            } else {
                tma_load_3d(bdst, &tmB, &full[s], k, int32_t(n0), ya);
            }
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = instr_desc(fmt<T>(), 128, BN, 0, r.b_mn ? 1u : 0u);
        bool ok = true;
        for (int64_t i = 0; i < nkb; ++i) {
            const int s = int(i % S);
            if (!mbar_wait(&full[s], uint32_t((i / S) & 1), abort, r.err, ERR_TIMEOUT_BASE + 2)) { ok = false; break; }
            tc_fence_after();
            if (r.dbg && i == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
                printf("[gemm dbg] nkb %lld kb %lld A0 %08x %08x B0 %08x %08x\n", (long long)nkb, (long long)kb,
                       reinterpret_cast<const uint32_t*>(As)[0], reinterpret_cast<const uint32_t*>(As)[1],
                       reinterpret_cast<const uint32_t*>(Bs)[0], reinterpret_cast<const uint32_t*>(Bs)[1]);
            const uint32_t a0 = smem_u32(As + s * a_bytes<T, BN>());
            const uint32_t b0 = smem_u32(Bs + s * b_bytes<T, BN>());
            for (int kk = 0; kk < BK / kInstK; ++kk) {
                const uint64_t ad = smem_desc(a0 + kk * 32, 16, 1024, 2);
                // B MN-major: column groups BK*128 bytes apart (LBO), K-row groups SBO apart:
                // 8 rows / 1024 B with the 16-byte swizzle atoms of 16-bit types; for 32-bit
                // (tf32) operands the MN-major layout uses 32-byte atoms, 4-row groups (512 B).
                constexpr bool kA32 = sizeof(T) == 4;
                const uint64_t bd = r.b_mn ? smem_desc(b0 + kk * (kInstK * 128), BK * 128, kA32 ? 512 : 1024,
                                                       kA32 ? 1 : 2)
                                           : smem_desc(b0 + kk * 32, 16, 1024, 2);
                if constexpr (std::is_same<T, float>::value) mma_ss_tf32(tmem, ad, bd, idesc, (i | kk) ? 1u : 0u);
                else mma_ss(tmem, ad, bd, idesc, (i | kk) ? 1u : 0u);
            }
            mma_commit(&empty[s]);
        }
        if (ok) mma_commit(acc_full);
    } else if (warp >= 2) {
        const int q = warp & 3;                       // TMEM lane quadrant of this warp
        const int row = q * 32 + lane;
        const int64_t m = m0 + row;
        bool ok = true;
        if (nkb > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort, r.err, ERR_TIMEOUT_BASE + 3));
            tc_fence_after();
        }
        if (ok) {
            const uint32_t lane_off = uint32_t(q * 32) << 16;
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                if (nkb > 0) {
                    tmem_ld32(tmem + lane_off + c * 32, v);
                    tmem_ld_wait();
                } else {
                    for (int e = 0; e < 32; ++e) v[e] = 0u;
                }
                const int64_t n = n0 + c * 32;
                if (r.dbg && c == 0 && row == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
                    printf("[gemm dbg] acc row0 %f %f  M %lld N %lld ldm %lld\n", __uint_as_float(v[0]),
                           __uint_as_float(v[1]), (long long)r.M, (long long)r.N, (long long)r.c_ldm);
                if (m >= r.M || n >= r.N) continue;
                const int64_t off = m * r.c_ldm + int64_t(z) * r.c_ldz + n;
                if (!r.c_is_t || std::is_same<T, float>::value) {
                    float4* d = reinterpret_cast<float4*>(static_cast<float*>(r.C) + off);
                    for (int e = 0; e < 8; ++e)
                        d[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                           __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
                } else {
                    uint4* d = reinterpret_cast<uint4*>(static_cast<T*>(r.C) + off);
                    for (int e = 0; e < 4; ++e) {
                        uint32_t w[4];
                        for (int h = 0; h < 4; ++h) {
                            const float lo = __uint_as_float(v[8 * e + 2 * h]), hi = __uint_as_float(v[8 * e + 2 * h + 1]);
                            if constexpr (std::is_same<T, __half>::value) {
                                __half2 h2 = __floats2half2_rn(lo, hi);
                                w[h] = *reinterpret_cast<uint32_t*>(&h2);
                            } else {
                                w[h] = pack_bf16(lo, hi);
                            }
                        }
                        d[e] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) { }
    }
    tc_fence_after();
    __syncwarp();
    if (warp == 1) tmem_dealloc(tmem, BN);
}

template <typename T, int BN>
mla_status_t launch(const TcGemm& g, cudaStream_t st) {
    constexpr int BK = tc_gemm_bk<T>();
    CUtensorMap ta, tb;
    const uint32_t abox[3] = {uint32_t(BK), 1u, 128u};
    const uint32_t bbox_mn[3] = {uint32_t(BK), uint32_t(BK), 1u};
    const uint32_t bbox_k[3] = {uint32_t(BK), uint32_t(BN), 1u};
    if (!make_map_3d<T>(&ta, g.A, g.a_dims, g.a_ld, abox, true) ||
        !make_map_3d<T>(&tb, g.B, g.b_dims, g.b_ld, g.b_mn ? bbox_mn : bbox_k, true,
                        /*atom32=*/g.b_mn && sizeof(T) == 4))
        return set_error(MLA_ERR_CUDA, "MLA: tensor map for the tensor-core GEMM failed (alignment?)");
    Run r{g.M, g.N, g.K, g.k_chunk, g.Z, g.split ? 1 : 0, g.b_mn ? 1 : 0, g.c_is_t ? 1 : 0, g.C, g.c_ldm, g.c_ldz,
          g.err, getenv("MLA_GEMM_DEBUG") ? 1 : 0};
    auto kern = tc_gemm_kernel<T, BN>;
    const size_t smem = smem_bytes<T, BN>();
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    dim3 grid(unsigned(ceil_div(g.N, BN)), unsigned(ceil_div(g.M, 128)), unsigned(g.Z));
    kern<<<grid, kThreads, smem, st>>>(ta, tb, r);
    return check_launch("tensor-core GEMM");
}

}  // namespace tcg

template <typename T>
mla_status_t tc_gemm(const TcGemm& g, cudaStream_t st) {
    if constexpr (std::is_same<T, double>::value) {
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: no fp64 tensor-core GEMM");
    } else {
        if (g.N % 32 != 0 || g.c_ldm % 8 != 0 || g.c_ldz % 8 != 0)
            return set_error(MLA_ERR_UNSUPPORTED, "MLA: tensor-core GEMM needs N, ldm, ldz multiples of 32/8");
        if (g.bn == 256) return tcg::launch<T, 256>(g, st);
        return tcg::launch<T, 128>(g, st);
    }
}

template mla_status_t tc_gemm<float>(const TcGemm&, cudaStream_t);
template mla_status_t tc_gemm<double>(const TcGemm&, cudaStream_t);
template mla_status_t tc_gemm<__half>(const TcGemm&, cudaStream_t);
template mla_status_t tc_gemm<__nv_bfloat16>(const TcGemm&, cudaStream_t);

}  // namespace mla
