// Tensor-core GEMM (tcgen05 + TMA) for the dense stages of the MLA forward.
//
// One CTA computes a 128 x BN output tile of one launch index z: warp 0 issues
// TMA loads of 128B-swizzled A and B blocks into a ring of stages, warp 1 (one
// thread) issues the MMAs (M = 128, N = BN, K = 8 tf32 or 16 bf16/fp16 per
// instruction) into a TMEM accumulator, warps 2-5 read the accumulator back
// (one TMEM lane = one output row per thread) and store it. With split3 (3xTF32,
// fp32 operands) warps 2-5 first split every landed stage into tf32 heads (in
// place) and fp32 remainders, and the MMA thread issues three MMAs per k-step.
// At decode batch sizes the projections are bound by HBM bandwidth on their
// weights, which every tile streams once.
#include "tc_gemm.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cstdio>
#include <cstdlib>

namespace mla {
namespace tcg {

using namespace sm100;

constexpr int kThreads = 192;
// 3xTF32 form of the one-tile kernel: warps 6-9 split the landed stages while
// warps 2-5 drain the accumulator, so neither waits for the other
template <bool S3> constexpr int kernel_threads() { return S3 ? 320 : kThreads; }
// 3xTF32: K blocks (32 elements each) summed into one TMEM accumulator before it is
// drained into the round-to-nearest running sum. Measured against fp64 on the
// attention fixtures: 1 block per drain matches fp32 CPU accuracy (rel-L2 7e-7),
// 2 blocks double the error, 4 blocks triple it.
#ifndef MLA_3XTF32_GROUP
#define MLA_3XTF32_GROUP 1
#endif
constexpr int kGroup = MLA_3XTF32_GROUP;
enum : int { ERR_TIMEOUT_BASE = 200 };

struct Run {
    int64_t M, N, K, k_chunk;
    int Z, spb, b_mn, c_is_t;
    int64_t nkb2;    // K blocks of the second operand pair (classic kernel only)
    float* rowmax; int64_t n_valid;   // classic kernel: per-row max of each tile's columns < n_valid
    void* C; int64_t c_ldm, c_ldz;
    int* err;
};

// fp32 -> tf32 rounded to nearest (ties away), as a 32-bit pattern
__device__ __forceinline__ uint32_t tf32_rna(uint32_t x) {
    uint32_t y;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(y) : "f"(__uint_as_float(x)));
    return y;
}

template <typename T> constexpr uint32_t fmt() {
    return std::is_same<T, float>::value ? 2u : std::is_same<T, __half>::value ? 0u : 1u;
}

// Stage counts: BN = 128 keeps 3 stages (97 KB) so two CTAs share an SM (a
// 192-CTA launch runs in one wave on 148 SMs); 3xTF32 stages also hold the
// remainders, so they are twice as large.
template <int BN, bool S3> constexpr int stages() { return S3 ? (BN == 256 ? 2 : 3) : (BN == 256 ? 4 : 3); }
constexpr int a_bytes() { return 128 * 128; }                     // 128 rows x 128 B
template <int BN> constexpr int b_bytes() { return BN * 128; }   // BN x one 128-byte K block
template <int BN, bool S3> constexpr size_t smem_bytes() {
    return 1024 + size_t(stages<BN, S3>()) * (a_bytes() + b_bytes<BN>()) * (S3 ? 2 : 1) + 512;
}

template <typename T, int BN, bool S3>
__global__ void __launch_bounds__(kernel_threads<S3>(), 1) tc_gemm_kernel(
    const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
    const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2, const Run r,
    const __grid_constant__ CUtensorMap tmC, const int use_tma_c)
{
    constexpr int S = stages<BN, S3>();
    constexpr int BK = tc_gemm_bk<T>();             // elements per 128-byte row
    constexpr int kInstK = 32 / int(sizeof(T));      // K per MMA instruction (32 bytes)
    constexpr int kStage = a_bytes() + b_bytes<BN>();
    // 3xTF32: two accumulators of BN columns (ping-pong over groups of kGroup K blocks),
    // a running sum at 2*BN, and two slots of the split A operand (tf32 hi | lo, one
    // 32-wide K block each: 64 columns) at kTmemA, read by ts-form MMAs
    constexpr uint32_t kTmemCols = S3 ? 512u : uint32_t(BN);
    static_assert(!S3 || BN == 128, "3xTF32 uses 128-column tiles");
    constexpr uint32_t kTmemA = 3u * BN;                 // 384: 2 slots x (32 hi + 32 lo) columns
    static_assert(!S3 || std::is_same<T, float>::value, "3xTF32 needs fp32 operands");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // stage s: [A | B] at smem + s*kStage; 3xTF32 remainders at lo + s*kStage
    unsigned char* lo = smem + S * kStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kStage * (S3 ? 2 : 1));
    uint64_t* empty = full + S;
    uint64_t* split_done = empty + S;
    uint64_t* acc_full = split_done + S;          // [2]: accumulator buffer ready (3xTF32 uses both)
    uint64_t* acc_empty = acc_full + 2;           // [2]: 3xTF32 accumulator drained into the sum
    uint64_t* a_free = acc_empty + 2;             // [2]: 3xTF32 TMEM A slot read by its MMAs
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_free + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    volatile int* abort = abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n0 = int64_t(blockIdx.x) * BN;
    const int64_t m0 = int64_t(blockIdx.y) * 128;
    const int z = blockIdx.z;
    const int ya = z / r.spb;                       // batch
    const int64_t kb = int64_t(z % r.spb) * r.k_chunk;
    const int64_t ke = min(r.K, kb + r.k_chunk);
    const int64_t nkb1 = ke > kb ? (ke - kb + BK - 1) / BK : 0;
    const int64_t nkb = nkb1 + r.nkb2;              // second operand pair (A2, B2) after the first

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
            mbar_init(&split_done[i], 128);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
            mbar_init(&a_free[i], 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (r.nkb2 > 0) {
            tma_prefetch_desc(&tmA2);
            tma_prefetch_desc(&tmB2);
        }
        for (int64_t i = 0; i < nkb; ++i) {
            const int s = int(i % S);
            if (!mbar_wait(&empty[s], uint32_t(((i / S) & 1) ^ 1), abort, r.err, ERR_TIMEOUT_BASE + 1)) break;
            const bool second = i >= nkb1;
            const CUtensorMap* ma = second ? &tmA2 : &tmA;
            const CUtensorMap* mb = second ? &tmB2 : &tmB;
            const int32_t k = second ? int32_t((i - nkb1) * BK) : int32_t(kb + i * BK);
            unsigned char* st = smem + s * kStage;
            mbar_arrive_expect_tx(&full[s], uint32_t(kStage));
            tma_load_3d(st, ma, &full[s], k, ya, int32_t(m0));
            unsigned char* bdst = st + a_bytes();
            if (r.b_mn) {
                for (int g = 0; g < BN / BK; ++g)   // BK-wide column groups of N, BK rows of K each
                    tma_load_3d(bdst + g * (BK * 128), mb, &full[s], int32_t(n0 + g * BK), k, ya);
            } else {
                tma_load_3d(bdst, mb, &full[s], k, int32_t(n0), ya);
            }
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = instr_desc(fmt<T>(), 128, BN, 0, r.b_mn ? 1u : 0u);
        bool ok = true;
        for (int64_t i = 0; i < nkb; ++i) {
            const int s = int(i % S);
            uint64_t* ready = S3 ? &split_done[s] : &full[s];
            if (!mbar_wait(ready, uint32_t((i / S) & 1), abort, r.err, ERR_TIMEOUT_BASE + 2)) { ok = false; break; }
            uint32_t d = tmem;
            bool fresh = i == 0;
            if constexpr (S3) {
                const int64_t gi = i / kGroup;
                d = tmem + uint32_t(gi & 1) * BN;
                fresh = i % kGroup == 0;
                if (fresh && !mbar_wait(&acc_empty[gi & 1], uint32_t(((gi >> 1) & 1) ^ 1), abort, r.err,
                                        ERR_TIMEOUT_BASE + 5)) { ok = false; break; }
            }
            tc_fence_after();
            const uint32_t a_hi = tmem + kTmemA + uint32_t(i & 1) * 64u;   // 3xTF32: split A in TMEM
            const uint32_t a0 = smem_u32(smem + s * kStage);
            const uint32_t b0 = a0 + a_bytes();
            // B MN-major: column groups BK*128 bytes apart (LBO), K-row groups SBO apart:
            // 8 rows / 1024 B with the 16-byte swizzle atoms of 16-bit types; for 32-bit
            // (tf32) operands the MN-major layout uses 32-byte atoms, 4-row groups (512 B).
            constexpr bool kA32 = sizeof(T) == 4;
            const uint64_t ad0 = smem_desc(a0, 16, 1024, 2);
            const uint64_t bd0 = r.b_mn ? smem_desc(b0, BK * 128, kA32 ? 512 : 1024, kA32 ? 1 : 2)
                                        : smem_desc(b0, 16, 1024, 2);
            const uint64_t lo_off = uint64_t((S * kStage) >> 4);   // remainder copy, same layout
#pragma unroll
            for (int kk = 0; kk < BK / kInstK; ++kk) {
                const uint64_t ad = ad0 + uint64_t((kk * 32) >> 4);
                const uint64_t bd = bd0 + uint64_t((r.b_mn ? kk * (kInstK * 128) : kk * 32) >> 4);
                const uint32_t acc = (fresh && kk == 0) ? 0u : 1u;
                if constexpr (std::is_same<T, float>::value) {
                    if constexpr (S3) {   // small terms first; A halves from TMEM
                        mma_ts_tf32(d, a_hi + kk * 8, bd + lo_off, idesc, acc);      // hi * lo
                        mma_ts_tf32(d, a_hi + 32 + kk * 8, bd, idesc, 1u);           // lo * hi
                        mma_ts_tf32(d, a_hi + kk * 8, bd, idesc, 1u);                // hi * hi
                    } else {
                        mma_ss_tf32(d, ad, bd, idesc, acc);
                    }
                } else {
                    mma_ss(d, ad, bd, idesc, acc);
                }
            }
            mma_commit(&empty[s]);
            if constexpr (S3) {
                mma_commit(&a_free[i & 1]);
                if ((i + 1) % kGroup == 0 || i + 1 == nkb) mma_commit(&acc_full[(i / kGroup) & 1]);
            }
        }
        if (ok && !S3) mma_commit(acc_full);
    } else if (S3 && warp >= 6) {
        // ------------------------------------------------------------ 3xTF32 split
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const uint32_t lane_off = uint32_t(q * 32) << 16;
        const int ts = threadIdx.x - 192;
        bool ok = true;
        for (int64_t i = 0; i < nkb && ok; ++i) {
            const int s = int(i % S);
            ok = __all_sync(0xffffffffu, mbar_wait(&full[s], uint32_t((i / S) & 1), abort, r.err,
                                                   ERR_TIMEOUT_BASE + 4));
            if (!ok) break;
            // A: my row (= my TMEM lane) of the 32-wide K block, split into the
            // TMEM slot of this block once its previous MMAs have read it
            ok = __all_sync(0xffffffffu, mbar_wait(&a_free[i & 1], uint32_t(((i >> 1) & 1) ^ 1), abort, r.err,
                                                   ERR_TIMEOUT_BASE + 7));
            if (!ok) break;
            tc_fence_after();
            {
                const unsigned char* arow = smem + s * kStage + row * 128;
                uint32_t h[32], l[32];
#pragma unroll
                for (int c = 0; c < 8; ++c) {   // 16-byte chunk c sits at c ^ (row % 8) (128B swizzle)
                    const uint4 v = *reinterpret_cast<const uint4*>(arow + ((c ^ (row & 7)) << 4));
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        h[4 * c + e] = tf32_rna(w[e]);
                        l[4 * c + e] = tf32_rna(__float_as_uint(__uint_as_float(w[e]) - __uint_as_float(h[4 * c + e])));
                    }
                }
                const uint32_t a_slot = tmem + lane_off + kTmemA + uint32_t(i & 1) * 64u;
                tmem_st32(a_slot, h);
                tmem_st32(a_slot + 32, l);
            }
            // B: hi in place, lo into the remainder buffer
            uint4* x = reinterpret_cast<uint4*>(smem + s * kStage + a_bytes());
            uint4* y = reinterpret_cast<uint4*>(lo + s * kStage + a_bytes());
#pragma unroll 4
            for (int e = ts; e < b_bytes<BN>() / 16; e += 128) {
                uint4 v = x[e], h, l;
                h.x = tf32_rna(v.x); h.y = tf32_rna(v.y); h.z = tf32_rna(v.z); h.w = tf32_rna(v.w);
                l.x = __float_as_uint(__uint_as_float(v.x) - __uint_as_float(h.x));
                l.y = __float_as_uint(__uint_as_float(v.y) - __uint_as_float(h.y));
                l.z = __float_as_uint(__uint_as_float(v.z) - __uint_as_float(h.z));
                l.w = __float_as_uint(__uint_as_float(v.w) - __uint_as_float(h.w));
                l.x = tf32_rna(l.x); l.y = tf32_rna(l.y); l.z = tf32_rna(l.z); l.w = tf32_rna(l.w);
                x[e] = h;
                y[e] = l;
            }
            tmem_st_wait();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&split_done[s]);
        }
    } else if (warp >= 2 && warp < 6) {
        const int q = warp & 3;                       // TMEM lane quadrant of this warp
        const int row = q * 32 + lane;
        const int64_t m = m0 + row;
        bool ok = true;
        const uint32_t lane_off = uint32_t(q * 32) << 16;
        uint32_t res = tmem;                          // accumulator the output is read from
        if constexpr (S3) {
            // split each landed stage: x = hi + lo with hi = x rounded to the nearest tf32
            // (kept in place) and lo = x - hi (exact in fp32), itself rounded to tf32, so
            // both halves carry unbiased rounding errors (truncation doubles the error).
            // The tensor core's fp32 accumulation does not round to nearest, so its error
            // grows with the number of MMAs summed into one accumulator: every kGroup K
            // blocks the accumulator is drained into a running sum (fp32, round to
            // nearest) kept in TMEM columns [2*BN, 3*BN).
            const int64_t ngroups = (nkb + kGroup - 1) / kGroup;
            auto harvest = [&](int64_t gi) -> bool {
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[gi & 1], uint32_t((gi >> 1) & 1), abort, r.err,
                                                       ERR_TIMEOUT_BASE + 6)))
                    return false;
                tc_fence_after();
                const uint32_t src = tmem + lane_off + uint32_t(gi & 1) * BN;
                const uint32_t sum = tmem + lane_off + 2u * BN;
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(src + c * 32, v);
                    if (gi > 0) {
                        uint32_t u[32];
                        tmem_ld32(sum + c * 32, u);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) + __uint_as_float(u[e]));
                    } else {
                        tmem_ld_wait();
                    }
                    tmem_st32(sum + c * 32, v);
                }
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&acc_empty[gi & 1]);
                return true;
            };

            for (int64_t gi = 0; gi < ngroups && ok; ++gi) ok = harvest(gi);

            res = tmem + 2u * BN;
        } else {
            if (ok && nkb > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort, r.err, ERR_TIMEOUT_BASE + 3));
                tc_fence_after();
            }
        }
        if (ok) {
            float rmax = -__int_as_float(0x7f800000);
            const bool leader = threadIdx.x == 64;   // issues the output TMA stores
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                if (nkb > 0) {
                    tmem_ld32(res + lane_off + c * 32, v);
                    tmem_ld_wait();
                } else {
                    for (int e = 0; e < 32; ++e) v[e] = 0u;
                }
                const int64_t n = n0 + c * 32;
                if (use_tma_c) {
                    // fp32 output through shared memory: every stage has been consumed
                    // (the accumulator is final), so two 16 KB buffers at the start of the
                    // stage area hold 128 x 32 chunks (row = thread, 128B swizzle), each
                    // leaving in one TMA store; rows and columns outside C are clipped
                    if (n >= r.N) continue;                       // same for every thread
                    if (r.rowmax)
                        for (int e = 0; e < 32; ++e)
                            if (n + e < r.n_valid) rmax = fmaxf(rmax, __uint_as_float(v[e]));
                    unsigned char* sbuf = smem + (c & 1) * (128 * 32 * 4);
                    if (leader) bulk_wait_read<1>();
                    named_bar_sync(1, 128);
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        *reinterpret_cast<uint4*>(sbuf + row * 128 + ((u ^ (row & 7)) << 4)) =
                            make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                    fence_proxy_async_smem();
                    named_bar_sync(1, 128);
                    if (leader) {
                        tma_store_3d(&tmC, sbuf, int32_t(n), int32_t(z), int32_t(m0));
                        bulk_commit();
                    }
                    continue;
                }
                if (m >= r.M || n >= r.N) continue;
                const int64_t off = m * r.c_ldm + int64_t(z) * r.c_ldz + n;
                if (!r.c_is_t || std::is_same<T, float>::value) {
                    float4* d = reinterpret_cast<float4*>(static_cast<float*>(r.C) + off);
                    for (int e = 0; e < 8; ++e) {
                        float4 o = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                               __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
                        d[e] = o;
                        if (r.rowmax) {
                            const float f[4] = {o.x, o.y, o.z, o.w};
                            for (int h = 0; h < 4; ++h)
                                if (n + 4 * e + h < r.n_valid) rmax = fmaxf(rmax, f[h]);
                        }
                    }
                } else {
                    uint4* d = reinterpret_cast<uint4*>(static_cast<T*>(r.C) + off);
                    for (int e = 0; e < 4; ++e) {
                        uint32_t w[4];
                        for (int h = 0; h < 4; ++h) {
                            const float lo_ = __uint_as_float(v[8 * e + 2 * h]), hi = __uint_as_float(v[8 * e + 2 * h + 1]);
                            if constexpr (std::is_same<T, __half>::value) {
                                __half2 h2 = __floats2half2_rn(lo_, hi);
                                w[h] = *reinterpret_cast<uint32_t*>(&h2);
                            } else {
                                w[h] = pack_bf16(lo_, hi);
                            }
                        }
                        d[e] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
            if (r.rowmax && m < r.M) r.rowmax[(int64_t(z) * r.M + m) * gridDim.x + blockIdx.x] = rmax;
            if (leader && use_tma_c) bulk_wait<0>();   // the output is written before the CTA retires
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
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------ persistent form
// One CTA per SM walks the output tiles (units) u = blockIdx.x, +gridDim.x, ...
// (N tile fastest, then M tile, then launch index z). The shared-memory ring runs
// on across units, and the accumulator is double-buffered in TMEM (2 x BN
// columns), so the epilogue of one unit overlaps the loads and MMAs of the next.
template <int BN> constexpr int pstages() { return BN == 256 ? 4 : BN == 192 ? 5 : 6; }
// fp32 output tiles leave through shared memory: two 128-row x 32-column fp32
// staging buffers (128B-swizzled), each stored by one TMA bulk tensor store
constexpr int kCStageBytes = 128 * 32 * 4;
// 192-column tiles serve only the RoPE epilogue (no fp32 C), so they keep no staging
template <int BN> constexpr int cstage_bytes() { return BN == 192 ? 0 : 2 * kCStageBytes; }
// RoPE epilogue: cos / sin of every (query, frequency) computed once per CTA
// when the queries are few (decode: every row of a tile shares one position)
constexpr int kRopeTabQ = 4;
template <int BN> constexpr int ropetab_bytes() { return BN == 192 ? kRopeTabQ * 64 * 8 : 0; }
// TMEM allocations are powers of two: two 192-column accumulators take 512 columns
template <int BN> constexpr uint32_t ptmem_cols() { return BN == 192 ? 512u : 2u * BN; }
template <int BN> constexpr size_t psmem_bytes() {
    return 1024 + size_t(pstages<BN>()) * (a_bytes() + b_bytes<BN>()) + cstage_bytes<BN>() + ropetab_bytes<BN>() +
           256;
}

struct Units {
    int64_t nt, mt, total;   // N tiles, M tiles, all units
};

template <typename T, int BN>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_persist_kernel(
    const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Run r, const Units U,
    const __grid_constant__ GemmRopeEpilogue re, const int use_re, const __grid_constant__ CUtensorMap tmC,
    const int use_tma_c)
{
    constexpr int S = pstages<BN>();
    constexpr int BK = tc_gemm_bk<T>();
    constexpr int kInstK = 32 / int(sizeof(T));
    constexpr int kStage = a_bytes() + b_bytes<BN>();
    constexpr uint32_t kTmemCols = ptmem_cols<BN>();
    static_assert(kStage % 1024 == 0, "stages stay 1024-byte aligned (128B swizzle)");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* cstage = smem + S * kStage;   // [2][kCStageBytes], 1024-aligned (not for BN 192)
    // (cos, sin) of positions[q] * inv_freq[j], [kRopeTabQ][64] (192-column tiles only)
    float2 (*rope_cs)[64] = reinterpret_cast<float2 (*)[64]>(cstage + cstage_bytes<BN>());
    uint64_t* full = reinterpret_cast<uint64_t*>(cstage + cstage_bytes<BN>() + ropetab_bytes<BN>());
    uint64_t* empty = full + S;
    uint64_t* acc_full = empty + S;     // [2]
    uint64_t* acc_empty = acc_full + 2; // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    volatile int* abort = abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // unit u -> (z, m0, n0) and its K range
    auto unit = [&](int64_t u, int& z, int64_t& m0, int64_t& n0, int64_t& kb, int64_t& nkb) {
        const int64_t per_z = U.nt * U.mt;
        z = int(u / per_z);
        const int64_t rem = u - int64_t(z) * per_z;
        m0 = (rem / U.nt) * 128;
        n0 = (rem % U.nt) * BN;
        kb = int64_t(z % r.spb) * r.k_chunk;
        const int64_t ke = min(r.K, kb + r.k_chunk);
        nkb = ke > kb ? (ke - kb + BK - 1) / BK : 0;
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (use_tma_c) tma_prefetch_desc(&tmC);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();      // the operands and the output may belong to the previous kernel
    pdl_trigger();

    if (warp == 0 && lane == 0) {
        int64_t it = 0;                      // k blocks issued so far (ring position)
        bool ok = true;
        for (int64_t u = blockIdx.x; u < U.total && ok; u += gridDim.x) {
            int z; int64_t m0, n0, kb, nkb;
            unit(u, z, m0, n0, kb, nkb);
            const int ya = z / r.spb;
            for (int64_t i = 0; i < nkb; ++i, ++it) {
                const int s = int(it % S);
                if (!mbar_wait(&empty[s], uint32_t(((it / S) & 1) ^ 1), abort, r.err, ERR_TIMEOUT_BASE + 11)) {
                    ok = false;
                    break;
                }
                const int32_t k = int32_t(kb + i * BK);
                unsigned char* st = smem + s * kStage;
                mbar_arrive_expect_tx(&full[s], uint32_t(kStage));
                tma_load_3d(st, &tmA, &full[s], k, ya, int32_t(m0));
                unsigned char* bdst = st + a_bytes();
                if (r.b_mn) {
                    for (int g = 0; g < BN / BK; ++g)
                        tma_load_3d(bdst + g * (BK * 128), &tmB, &full[s], int32_t(n0 + g * BK), k, ya);
                } else {
                    tma_load_3d(bdst, &tmB, &full[s], k, int32_t(n0), ya);
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        const uint32_t idesc = instr_desc(fmt<T>(), 128, BN, 0, r.b_mn ? 1u : 0u);
        constexpr bool kA32 = sizeof(T) == 4;
        int64_t it = 0, lt = 0;
        bool ok = true;
        for (int64_t u = blockIdx.x; u < U.total && ok; u += gridDim.x, ++lt) {
            int z; int64_t m0, n0, kb, nkb;
            unit(u, z, m0, n0, kb, nkb);
            const int buf = int(lt & 1);
            if (!mbar_wait(&acc_empty[buf], uint32_t(((lt >> 1) & 1) ^ 1), abort, r.err, ERR_TIMEOUT_BASE + 12)) break;
            tc_fence_after();
            const uint32_t d = tmem + uint32_t(buf) * BN;
            for (int64_t i = 0; i < nkb; ++i, ++it) {
                const int s = int(it % S);
                if (!mbar_wait(&full[s], uint32_t((it / S) & 1), abort, r.err, ERR_TIMEOUT_BASE + 13)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(smem + s * kStage);
                const uint32_t b0 = a0 + a_bytes();
                const uint64_t ad0 = smem_desc(a0, 16, 1024, 2);
                const uint64_t bd0 = r.b_mn ? smem_desc(b0, BK * 128, kA32 ? 512 : 1024, kA32 ? 1 : 2)
                                            : smem_desc(b0, 16, 1024, 2);
#pragma unroll
                for (int kk = 0; kk < BK / kInstK; ++kk) {
                    const uint64_t ad = ad0 + uint64_t((kk * 32) >> 4);
                    const uint64_t bd = bd0 + uint64_t((r.b_mn ? kk * (kInstK * 128) : kk * 32) >> 4);
                    const uint32_t acc = (i | kk) ? 1u : 0u;
                    if constexpr (std::is_same<T, float>::value) mma_ss_tf32(d, ad, bd, idesc, acc);
                    else mma_ss(d, ad, bd, idesc, acc);
                }
                mma_commit(&empty[s]);
            }
            if (!ok) break;
            mma_commit(&acc_full[buf]);
        }
    } else if (warp >= 2) {
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const uint32_t lane_off = uint32_t(q * 32) << 16;
        const bool leader = threadIdx.x == 64;   // issues the output TMA stores
        uint32_t chunk = 0;                      // staging-buffer sequence
        int64_t lt = 0;
        const bool rope_tab = ropetab_bytes<BN>() > 0 && use_re && re.sq <= kRopeTabQ;
        if (rope_tab) {
            const int half = int(re.rope / 2);
            for (int idx = threadIdx.x - 64; idx < int(re.sq) * half; idx += 128) {
                const int qq = idx / half, j = idx % half;
                const float ang = float(re.positions[qq]) * re.inv_freq[j];
                rope_cs[qq][j] = make_float2(cosf(ang), sinf(ang));
            }
            named_bar_sync(1, 128);
        }
        for (int64_t u = blockIdx.x; u < U.total; u += gridDim.x, ++lt) {
            int z; int64_t m0, n0, kb, nkb;
            unit(u, z, m0, n0, kb, nkb);
            const int buf = int(lt & 1);
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], uint32_t((lt >> 1) & 1), abort, r.err,
                                                   ERR_TIMEOUT_BASE + 14)))
                break;
            tc_fence_after();
            const int64_t m = m0 + row;
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                if (nkb > 0) {
                    tmem_ld32(tmem + lane_off + uint32_t(buf) * BN + c * 32, v);
                    tmem_ld_wait();
                } else {
                    for (int e = 0; e < 32; ++e) v[e] = 0u;
                }
                const int64_t n = n0 + c * 32;
                if (use_tma_c) {
                    // stage the 128 x 32 chunk (row = thread, 128B swizzle), then one
                    // TMA store; the buffer is rewritten two chunks later, once that
                    // store has read it
                    if (n >= r.N) continue;                       // same for every thread
                    unsigned char* sb = cstage + (chunk & 1u) * kCStageBytes;
                    if (leader) bulk_wait_read<1>();
                    named_bar_sync(1, 128);
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        *reinterpret_cast<uint4*>(sb + row * 128 + ((u ^ (row & 7)) << 4)) =
                            make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                    fence_proxy_async_smem();
                    named_bar_sync(1, 128);
                    if (leader) {
                        tma_store_3d(&tmC, sb, int32_t(n), int32_t(z), int32_t(m0));
                        bulk_commit();
                    }
                    ++chunk;
                    continue;
                }
                if (m >= r.M || n >= r.N) continue;
                if (use_re) {   // 2a2 epilogue: split per head, RoPE on the rope part
                    const int64_t qk = re.nope + re.rope;
                    const int64_t h = n / qk, o = n - h * qk;
                    if (o < re.nope) {
                        uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(re.q_nope) +
                                                              (m * re.heads + h) * re.nope + o);
                        for (int e = 0; e < 4; ++e) {
                            uint32_t w[4];
                            for (int hh = 0; hh < 4; ++hh) {
                                const float lo_ = __uint_as_float(v[8 * e + 2 * hh]);
                                const float hi = __uint_as_float(v[8 * e + 2 * hh + 1]);
                                if constexpr (std::is_same<T, __half>::value) {
                                    __half2 h2 = __floats2half2_rn(lo_, hi);
                                    w[hh] = *reinterpret_cast<uint32_t*>(&h2);
                                } else {
                                    w[hh] = pack_bf16(lo_, hi);
                                }
                            }
                            dst[e] = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    } else {
                        const int64_t ro = o - re.nope;                 // first rope dim of this chunk
                        const int64_t qq = m % re.sq;
                        const float pos = float(re.positions[qq]);
                        float4* dst = reinterpret_cast<float4*>(re.q_rope + (m * re.heads + h) * re.rope + ro);
                        for (int e = 0; e < 8; ++e) {
                            float out[4];
                            for (int pp = 0; pp < 2; ++pp) {
                                const int j = int(ro / 2) + 2 * e + pp;
                                float cs, sn;
                                if (rope_tab) {
                                    const float2 t = rope_cs[qq][j];
                                    cs = t.x;
                                    sn = t.y;
                                } else {
                                    const float ang = pos * re.inv_freq[j];
                                    cs = cosf(ang);
                                    sn = sinf(ang);
                                }
                                const float ev = __uint_as_float(v[4 * e + 2 * pp]);
                                const float od = __uint_as_float(v[4 * e + 2 * pp + 1]);
                                out[2 * pp] = ev * cs - od * sn;
                                out[2 * pp + 1] = ev * sn + od * cs;
                            }
                            dst[e] = make_float4(out[0], out[1], out[2], out[3]);
                        }
                    }
                    continue;
                }
                const int64_t off = m * r.c_ldm + int64_t(z) * r.c_ldz + n;
                if (!r.c_is_t || std::is_same<T, float>::value) {
                    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(r.C) + off);
                    for (int e = 0; e < 8; ++e)
                        dst[e] = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                             __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
                } else {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(r.C) + off);
                    for (int e = 0; e < 4; ++e) {
                        uint32_t w[4];
                        for (int h = 0; h < 4; ++h) {
                            const float lo_ = __uint_as_float(v[8 * e + 2 * h]), hi = __uint_as_float(v[8 * e + 2 * h + 1]);
                            if constexpr (std::is_same<T, __half>::value) {
                                __half2 h2 = __floats2half2_rn(lo_, hi);
                                w[h] = *reinterpret_cast<uint32_t*>(&h2);
                            } else {
                                w[h] = pack_bf16(lo_, hi);
                            }
                        }
                        dst[e] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[buf]);
        }
        if (leader && use_tma_c) bulk_wait<0>();   // the output is written before the CTA retires
    }
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) { }
    }
    tc_fence_after();
    __syncwarp();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <typename T, int BN>
mla_status_t launch_persist(const TcGemm& g, cudaStream_t st) {
    constexpr int BK = tc_gemm_bk<T>();
    CUtensorMap ta, tb;
    const uint32_t abox[3] = {uint32_t(BK), 1u, 128u};
    const uint32_t bbox_mn[3] = {uint32_t(BK), uint32_t(BK), 1u};
    const uint32_t bbox_k[3] = {uint32_t(BK), uint32_t(BN), 1u};
    if (!make_map_3d<T>(&ta, g.A, g.a_dims, g.a_ld, abox, true) ||
        !make_map_3d<T>(&tb, g.B, g.b_dims, g.b_ld, g.b_mn ? bbox_mn : bbox_k, true,
                        /*atom32=*/g.b_mn && sizeof(T) == 4))
        return set_error(MLA_ERR_CUDA, "MLA: tensor map for the tensor-core GEMM failed (alignment?)");
    Run r{g.M, g.N, g.K, g.spb > 1 ? g.k_chunk : g.K, g.Z, g.spb > 1 ? g.spb : 1, g.b_mn ? 1 : 0,
          g.c_is_t ? 1 : 0, 0, nullptr, 0, g.C, g.c_ldm, g.c_ldz, g.err};
    Units U{ceil_div(g.N, BN), ceil_div(g.M, 128), 0};
    U.total = U.nt * U.mt * g.Z;
    auto kern = tc_gemm_persist_kernel<T, BN>;
    const size_t smem = psmem_bytes<BN>();
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    const int64_t grid = U.total < sm_count() ? U.total : sm_count();
    GemmRopeEpilogue re{};
    if (g.rope_epi) re = *g.rope_epi;
    // fp32 output: a map over C's (n, z, m) with box 32 x 1 x 128 for the TMA-store epilogue
    CUtensorMap tc{};
    int use_tma_c = 0;
    if (cstage_bytes<BN>() > 0 && !g.rope_epi && (!g.c_is_t || std::is_same<T, float>::value) &&
        (reinterpret_cast<uintptr_t>(g.C) & 15) == 0) {
        const int64_t cdims[3] = {g.N, g.Z, g.M};
        const int64_t cld[2] = {g.c_ldz, g.c_ldm};
        const uint32_t cbox[3] = {32u, 1u, 128u};
        use_tma_c = make_map_3d<float>(&tc, g.C, cdims, cld, cbox, true) ? 1 : 0;
    }
    launch_pdl(kern, dim3(unsigned(grid)), dim3(kThreads), smem, st, ta, tb, r, U, re, g.rope_epi ? 1 : 0, tc,
               use_tma_c);
    return check_launch("tensor-core GEMM (persistent)");
}

template <typename T, int BN, bool S3>
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
    CUtensorMap ta2 = ta, tb2 = tb;
    if (g.K2 > 0 &&
        (!make_map_3d<T>(&ta2, g.A2, g.a2_dims, g.a2_ld, abox, true) ||
         !make_map_3d<T>(&tb2, g.B2, g.b2_dims, g.b2_ld, g.b_mn ? bbox_mn : bbox_k, true,
                         /*atom32=*/g.b_mn && sizeof(T) == 4)))
        return set_error(MLA_ERR_CUDA, "MLA: tensor map for the tensor-core GEMM failed (alignment?)");
    Run r{g.M, g.N, g.K, g.spb > 1 ? g.k_chunk : g.K, g.Z, g.spb > 1 ? g.spb : 1, g.b_mn ? 1 : 0,
          g.c_is_t ? 1 : 0, g.K2 > 0 ? ceil_div(g.K2, BK) : 0,
          g.rowmax, g.rowmax ? g.n_valid : 0, g.C, g.c_ldm, g.c_ldz, g.err};
    auto kern = tc_gemm_kernel<T, BN, S3>;
    const size_t smem = smem_bytes<BN, S3>();
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    dim3 grid(unsigned(ceil_div(g.N, BN)), unsigned(ceil_div(g.M, 128)), unsigned(g.Z));
    // fp32 output: TMA-store epilogue over C's (n, z, m) map (box 32 x 1 x 128)
    CUtensorMap tc{};
    int use_tma_c = 0;
    if ((!g.c_is_t || std::is_same<T, float>::value) && (reinterpret_cast<uintptr_t>(g.C) & 15) == 0) {
        const int64_t cdims[3] = {g.N, g.Z, g.M};
        const int64_t cld[2] = {g.c_ldz, g.c_ldm};
        const uint32_t cbox[3] = {32u, 1u, 128u};
        use_tma_c = make_map_3d<float>(&tc, g.C, cdims, cld, cbox, true) ? 1 : 0;
    }
    kern<<<grid, kernel_threads<S3>(), smem, st>>>(ta, tb, ta2, tb2, r, tc, use_tma_c);
    return check_launch("tensor-core GEMM");
}

}  // namespace tcg

// MLA_GEMM_CLASSIC=1 (debug): one CTA per output tile instead of the persistent form.
static bool tc_gemm_classic() {
    static const bool v = getenv("MLA_GEMM_CLASSIC") != nullptr && getenv("MLA_GEMM_CLASSIC")[0] == '1';
    return v;
}

template <typename T>
mla_status_t tc_gemm(const TcGemm& g, cudaStream_t st) {
    if constexpr (std::is_same<T, double>::value) {
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: no fp64 tensor-core GEMM");
    } else {
        if (g.N % 32 != 0 || g.c_ldm % 8 != 0 || g.c_ldz % 8 != 0)
            return set_error(MLA_ERR_UNSUPPORTED, "MLA: tensor-core GEMM needs N, ldm, ldz multiples of 32/8");
        if (g.Z <= 0 || g.M <= 0) return MLA_OK;
        if constexpr (std::is_same<T, float>::value) {
            if (g.split3) return tcg::launch<T, 128, true>(g, st);
        } else {
            if (g.split3) return set_error(MLA_ERR_UNSUPPORTED, "MLA: 3xTF32 needs fp32 operands");
        }
        if (g.rope_epi) {
            const GemmRopeEpilogue& e = *g.rope_epi;
            if (g.spb != 1 || g.Z != 1 || e.nope % 32 || e.rope % 32 || e.rope / 2 > 64 ||
                g.N != e.heads * (e.nope + e.rope))
                return set_error(MLA_ERR_UNSUPPORTED, "MLA: RoPE epilogue needs no split-K and 32-aligned parts");
            if (g.bn == 256) return tcg::launch_persist<T, 256>(g, st);
            if (g.bn == 192) return tcg::launch_persist<T, 192>(g, st);
            return tcg::launch_persist<T, 128>(g, st);
        }
        if (g.K2 == 0 && !g.rowmax && !tc_gemm_classic()) {
            if (g.bn == 256) return tcg::launch_persist<T, 256>(g, st);
            if (g.bn == 192) return tcg::launch_persist<T, 192>(g, st);
            return tcg::launch_persist<T, 128>(g, st);
        }
        if (g.bn == 256) return tcg::launch<T, 256, false>(g, st);
        return tcg::launch<T, 128, false>(g, st);
    }
}

template mla_status_t tc_gemm<float>(const TcGemm&, cudaStream_t);
template mla_status_t tc_gemm<double>(const TcGemm&, cudaStream_t);
template mla_status_t tc_gemm<__half>(const TcGemm&, cudaStream_t);
template mla_status_t tc_gemm<__nv_bfloat16>(const TcGemm&, cudaStream_t);

}  // namespace mla
