// Tensor-core absorbed-MLA decode attention for sm_100a (MLA_PREC_TENSOR).
//
// Semantics: the reference's steps 3a-3c (mla_kernels.cu:808-1326, PyTorch
// path exhaustive_benchmark_suite.py:289-304) fused into one persistent
// flash-decode kernel, then an LSE combine of key segments and the W_uv
// up-projection (3d, mla_kernels.cu:1339-1476). Scores never reach memory.
//
// Work unit. A "group" is one (b, q): the 128 heads of query q of sequence b,
// which share the keys of sequence b. Each group is cut into 64-key tiles; all
// tiles of all groups are laid end to end and split evenly over the persistent
// clusters (stream-K), so every SM gets the same number of key tiles whatever
// B and Sk are. A cluster's tiles of one group form a "segment"; each segment
// leaves an unnormalised partial output plus its (max, sum) for the combine.
//
// Cluster of two CTAs (one per SM). The 576 score dims are split evenly
// between them: CTA r owns c_kv dims [256r, 256r+256) and rope dims
// [32r, 32r+32). Per key tile each CTA
//   * loads only its own dims of the tile (TMA), once from HBM;
//   * computes a partial score S_r = Q[:, dims_r] . K[:, dims_r]^T on the
//     tensor cores (M = 128 heads, N = 64 keys, K = 288) into TMEM;
//   * swaps S_r with its peer through distributed shared memory, in log2
//     units rounded to fp16; both CTAs round both halves the same way, so both
//     hold the same S = S_0 + S_1 and run the same online softmax;
//   * accumulates its half of the context, O_r += P . V[:, 256r:256r+256]
//     (M = 128, N = 256, K = 64) in TMEM. The same shared-memory tile is the
//     K-major B operand of the score MMA and the MN-major B operand of P.V.
// TMEM per CTA (512 columns): O half 256, two score / probability buffers of
// 64, the bf16 latent query slice 128 (A operand read from TMEM). The 32 rope
// dims of the query are an A operand in shared memory.
//
// Operands are bf16 (fp16 for fp16 storage) with fp32 accumulation. fp32
// storage is converted to bf16 in shared memory after the TMA load, so HBM
// traffic stays one read of the fp32 cache.
//
// Warp roles (640 threads): warp 0 TMA producer, warp 1 score-MMA issuer and
// TMEM owner, warp 2 P.V issuer (warp 3 idle), warps 16-19 fp32->bf16
// converters (fp32 storage only), warps
// 4-7 and 12-15 softmax (keys 0-31 / 32-63 of each tile), warps 8-11 exchange
// (query loads, partial-score push to the peer). Thread i of a warpgroup <->
// TMEM lane i <-> head i: a warp reaches only TMEM lanes 32*(warp%4)..+31.
#include "tc.cuh"
#include "sm100.cuh"
#include "tc_gemm.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unistd.h>
#include <type_traits>
#include <vector>
#include <algorithm>

namespace mla {

// Runs steps 3d from a normalised context (defined in attn_exact.cu).
template <typename T> mla_status_t attn_out_normalized(const AArgs& a, const float* O, cudaStream_t st);

namespace tc {

using namespace sm100;

constexpr int NK = 64;                      // keys per tile
constexpr int kHeads = 128;
constexpr int kRank = 512;
constexpr int kRope = 64;
constexpr int kHalf = 256;                  // latent dims per CTA
constexpr int kRopeHalf = 32;               // rope dims per CTA
constexpr int kThreads = 640;
constexpr int kQPrefetchTiles = 4;          // L2 prefetch of the next group's query, tiles ahead
// Registers per thread at launch. The per-warpgroup split below (setmaxnreg)
// is computed from it, and an increase waits until other warpgroups have
// released enough, so the host refuses to launch if the compiled kernel does
// not use exactly this many (a mismatch could leave an increase waiting).
constexpr int kLaunchRegs = 96;
// per-thread registers of each warpgroup after the split (see the kernel)
constexpr int kRegBase = 80, kRegSoftmax = 128, kRegExchange = 72, kRegConvert = 72;
static_assert(kRegBase + 2 * kRegSoftmax + kRegExchange + kRegConvert <= 5 * kLaunchRegs,
              "register split exceeds the launch allocation: setmaxnreg.inc would wait forever");
static_assert(kThreads == 5 * 128, "five warpgroups");
constexpr int kConvThreads = 128;           // fp32 -> bf16 converter threads (warps 16-19)
constexpr int kChunkBytes = NK * 128;       // 64 latent dims of a tile: 64 rows of 128 B, 128B swizzle
constexpr int kRopeChunkBytes = NK * 64;    // 32 rope dims of a tile: 64 rows of 64 B, 64B swizzle
constexpr int kSlotBytes = 4 * kChunkBytes + kRopeChunkBytes;
constexpr int kStgRows = 16;                // an fp32 staging buffer holds a quarter of a key tile
constexpr int kStgLatBytes = kStgRows * kHalf * 4;
constexpr int kStgBytes = kStgRows * (kHalf + kRopeHalf) * 4;
constexpr int kXBufs = 2;                   // partial-score exchange buffers (flow-controlled)
// one exchange buffer: the 128 rows x 64 partial scores of a tile, in log2 units
// (times log2(e)/scale) rounded to fp16, stored chunk-major (16-byte chunk e =
// keys 8e..8e+7 of row r at (e*128 + r)*16), so that a warp's 32 rows write and
// read 512 contiguous bytes per instruction
constexpr int kXBytesF16 = kHeads * NK * 2;
constexpr int kQRopeBytes = kHeads * kRopeHalf * 2;   // rope query slice: 128 rows of 64 B, 64B swizzle

// TMEM columns: O half, kSBufs score / probability buffers, the query slice.
constexpr uint32_t kTmemO = 0;
constexpr int kSBufs = 2;
constexpr uint32_t kTmemS = 256;
constexpr uint32_t kTmemQ = 256 + kSBufs * NK;   // 128 columns, ends at column 512
constexpr uint32_t kTmemCols = 512;
static_assert(kTmemQ + kHalf / 2 == kTmemCols, "TMEM budget");

enum : int { ERR_TIMEOUT_BASE = 100 };

template <typename T> struct Traits;
// Staging depth: fp32 tiles stream through kStages quarter-tile buffers, whose
// bytes are what the SM has in flight from HBM; four (a whole tile) cover the
// load latency at the tile rate the rest of the pipeline sustains.
template <> struct Traits<float> {
    static constexpr bool kConvert = true;
    static constexpr int kSlots = 3;
    static constexpr int kStages = 4;
    static constexpr uint32_t kFmt = 1;     // bf16 operands
};
template <> struct Traits<__nv_bfloat16> {
    static constexpr bool kConvert = false; static constexpr int kSlots = 5; static constexpr int kStages = 0;
    static constexpr uint32_t kFmt = 1;
};
template <> struct Traits<__half> {
    static constexpr bool kConvert = false; static constexpr int kSlots = 5; static constexpr int kStages = 0;
    static constexpr uint32_t kFmt = 0;     // fp16 operands
};

// Shared memory: kSlots 16-bit key tiles (the MMA operands: four 128B-swizzled
// latent chunks and one 64B-swizzled rope chunk each), kStages fp32
// quarter-tile staging buffers (fp32 storage only), the exchange buffers, the
// rope query slice, barriers. 16-bit storage is loaded by TMA straight into
// the slots; fp32 storage lands in staging, which the converter warps release
// as soon as they have read it (so TMA keeps loads in flight), and is
// converted into slots.
// Kernel configuration. kExact (16-bit storage only) is the exact-precision
// variant: the partial scores travel in fp32 (exchange buffers of 32 KB, one
// slot fewer), and P is split into a 16-bit head and remainder, P = P_hi + P_lo,
// both multiplied into V, so P.V carries the probabilities to about 2^-17
// relative (the reference multiplies fp32 probabilities into the 16-bit cache).
template <typename T, bool kExact> struct Cfg {
    static constexpr bool kConvert = Traits<T>::kConvert;
    static constexpr int kSlots = kExact ? 4 : Traits<T>::kSlots;
    static constexpr int kStages = Traits<T>::kStages;
    static constexpr uint32_t kFmt = Traits<T>::kFmt;
    static constexpr int kXBytes = kExact ? kHeads * NK * 4 : kXBytesF16;
};

template <typename T, bool kExact = false>
constexpr size_t smem_bytes() {
    using C = Cfg<T, kExact>;
    return 1024 /*align slack*/ + size_t(C::kSlots) * kSlotBytes + size_t(C::kStages) * kStgBytes +
           kXBufs * size_t(C::kXBytes) + kQRopeBytes + 4096 /*barriers, row maxima, row sums*/;
}
static_assert(smem_bytes<float>() <= 232448 && smem_bytes<__nv_bfloat16>() <= 232448 &&
              smem_bytes<__nv_bfloat16, true>() <= 232448, "shared memory budget");

struct Params {
    const void* qa;     // [B*Sq*H, 512]
    const void* qr;     // [B*Sq*H, 64]
    float* O_part;      // [slots][128 chunks of 4 dims][128 heads][4]: chunk-major, see the epilogue
    float* ml;          // [slots, 128, 2]  (running max in log2 units, sum)
    int* err;
    int* trace;         // debug only (MLA_TC_TRACE): per-CTA progress words in mapped host memory
    long long* prof;    // debug only (MLA_TC_PROFILE builds): [grid][kProfSlots] cycle counters
    long long* tl;      // debug only (MLA_TC_TIMELINE builds): [2 CTAs][kTlEvents][kTlTiles] clock64
    int64_t batch, sq, sk;
    int causal;
    float c_log2;       // log2(e) / scale
    int64_t total_tiles, tiles_per_cluster;
    int max_segs;
};

// Key tiles of group g = (b, q).
__device__ __forceinline__ int64_t group_keys(const Params& p, int64_t g) {
    if (!p.causal) return p.sk;
    const int64_t q = g % p.sq;
    return p.sk - p.sq + q + 1;
}
__device__ __forceinline__ int64_t group_tiles(const Params& p, int64_t g) {
    return (group_keys(p, g) + NK - 1) / NK;
}
// sum of ceil(x / NK) over x = 1..n (n >= 0): with n = NK*m + r, NK*m(m+1)/2 + r(m+1)
__device__ __forceinline__ int64_t ceil_sum(int64_t n) {
    if (n <= 0) return 0;
    const int64_t m = n / NK, r = n % NK;
    return (NK / 2) * m * (m + 1) + r * (m + 1);
}
// Key tiles of queries 0..q-1 of one sequence, in closed form (query i has
// sk - sq + 1 + i keys under causal masking, sk otherwise), so that locating a
// tile costs O(log sq) rather than a walk over every query (prefill has
// thousands).
__device__ __forceinline__ int64_t tiles_before(const Params& p, int64_t q) {
    if (!p.causal) return q * ((p.sk + NK - 1) / NK);
    const int64_t a = p.sk - p.sq + 1;   // keys of query 0 (>= 1: causal needs sk >= sq)
    return ceil_sum(a + q - 1) - ceil_sum(a - 1);
}

// Debug cycle accounting (compiled in with -DMLA_TC_PROFILE, printed by the host
// when MLA_TC_PROF is set): clock64 cycles spent in each wait site (slot = the
// site's timeout code - 100) and in a few work phases, summed per CTA.
#ifdef MLA_TC_PROFILE
#define MLA_TW(slot, expr) ([&]() { const long long _t0 = clock64(); const bool _r = (expr); \
    wacc[slot] += clock64() - _t0; return _r; }())
#define MLA_PROF(stmt) stmt
#else
#define MLA_TW(slot, expr) (expr)
#define MLA_PROF(stmt)
#endif
constexpr int kProfSlots = 26;
// Debug per-tile timeline (compiled in with -DMLA_TC_TIMELINE, printed by the
// host when MLA_TC_TL is set): clock64 of eight pipeline events for the first
// kTlTiles tiles of CTAs 0 and 1.
constexpr int kTlTiles = 256;
constexpr int kTlEvents = 12;
#ifdef MLA_TC_TIMELINE
#define MLA_TL(ev, i) do { if (p.tl && blockIdx.x < 2 && (i) < kTlTiles) \
    p.tl[(blockIdx.x * kTlEvents + (ev)) * kTlTiles + (i)] = clock64(); } while (0)
#else
#define MLA_TL(ev, i) do { } while (0)
#endif

__device__ __forceinline__ void trace_put(const Params& p, int role, int64_t v) {
    if (p.trace) *reinterpret_cast<volatile int*>(p.trace + blockIdx.x * 32 + role) = int(v);
}

struct TileIter {
    int64_t g, j, tiles, keys;
};

// Locates global tile index t: returns the group and the tile inside it.
__device__ __forceinline__ TileIter locate(const Params& p, int64_t t) {
    const int64_t per_batch = tiles_before(p, p.sq);
    const int64_t b = t / per_batch;
    const int64_t r = t % per_batch;
    int64_t lo = 0, hi = p.sq - 1;   // the last query whose first tile is at or before r
    while (lo < hi) {
        const int64_t mid = (lo + hi + 1) / 2;
        if (tiles_before(p, mid) <= r) lo = mid; else hi = mid - 1;
    }
    TileIter it;
    it.g = b * p.sq + lo;
    it.j = r - tiles_before(p, lo);
    it.keys = group_keys(p, it.g);
    it.tiles = (it.keys + NK - 1) / NK;
    return it;
}
__device__ __forceinline__ void advance(const Params& p, TileIter& it) {
    if (++it.j == it.tiles) {
        ++it.g;
        it.j = 0;
        it.keys = group_keys(p, it.g);
        it.tiles = (it.keys + NK - 1) / NK;
    }
}

struct Bars {
    uint64_t full[6];         // TMA data landed: slots (16-bit) or staging buffers (fp32)
    uint64_t stg_empty[6];    // fp32: staging buffer read by all converter threads
    uint64_t bf_full[6];      // fp32: converted slot ready
    uint64_t bf_empty[6];     // slot released by the P.V MMA
    uint64_t s_full[kSBufs];
    uint64_t p_full[kSBufs];
    uint64_t o_done[kSBufs];
    uint64_t x_full[kXBufs][4];   // per softmax warp: peer's partial scores arrived (st.async byte count)
    uint64_t x_free[kXBufs][4];   // per exchange warp: the peer has read my previous push into its buffer
                                  // (completed by a 4-byte st.async from the peer's softmax warp)
    float sink[kXBufs][4];        // landing words of those 4-byte signals
    float xmax[2][2 * kHeads];    // per tile parity: the two softmax warps' half-tile row maxima
    float xl[2 * kHeads];         // epilogue: the two softmax warps' partial row sums
    uint64_t s_read[kSBufs];      // the exchange warps have read my partial scores of the buffer
    uint64_t q_ready;
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(Bars) <= 4096, "barrier area");
static_assert(Traits<float>::kSlots <= 6 && Traits<float>::kStages <= 6 && Traits<__nv_bfloat16>::kSlots <= 6 &&
              Traits<__half>::kSlots <= 6, "barrier arrays");

// 64B-swizzled byte offset of 16-byte unit u (0..3) of row r in a region of
// 64-byte rows (the layout TMA's SWIZZLE_64B writes and the MMA descriptor's
// 64-byte swizzle mode reads).
__device__ __forceinline__ uint32_t swz64(uint32_t r, uint32_t u) { return r * 64u + ((u ^ ((r >> 1) & 3u)) << 4); }
// 128B-swizzled byte offset of 16-byte unit u (0..7) of row r (128-byte rows).
__device__ __forceinline__ uint32_t swz128(uint32_t r, uint32_t u) { return r * 128u + ((u ^ (r & 7u)) << 4); }

// Two partial scores in log2 units (times c = log2(e)/scale), rounded to fp16
// (finite: saturates at +-65504) and packed (lo, hi). Both CTAs of a pair round
// their own and the peer's partial the same way, so both hold the same sums.
__device__ __forceinline__ uint32_t pack_x16(float lo, float hi, float c) {
    uint32_t d;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi * c), "f"(lo * c));
    return d;
}
__device__ __forceinline__ float2 unpack_x16(uint32_t v) {
    __half2 h;
    memcpy(&h, &v, 4);
    return __half22float2(h);
}

template <typename T, bool kExact>
__global__ void __maxnreg__(kLaunchRegs) mla_decode_tc_kernel(
    const __grid_constant__ CUtensorMap tm_ckv, const __grid_constant__ CUtensorMap tm_pe, const Params p)
{
    using Tr = Cfg<T, kExact>;
    static_assert(!kExact || !Traits<T>::kConvert, "the exact variant is for 16-bit storage");
    constexpr int kXB = Tr::kXBytes;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* slots = smem;
    unsigned char* stg = slots + Tr::kSlots * kSlotBytes;
    float* xbuf = reinterpret_cast<float*>(stg + Tr::kStages * kStgBytes);
    unsigned char* qrope = reinterpret_cast<unsigned char*>(xbuf) + kXBufs * kXB;
    Bars* bars = reinterpret_cast<Bars*>(qrope + kQRopeBytes);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const int64_t cl = cluster_id_x();
    const int64_t t_begin = cl * p.tiles_per_cluster;
    const int64_t t_end = min(t_begin + p.tiles_per_cluster, p.total_tiles);
    const int64_t n = t_end > t_begin ? t_end - t_begin : 0;   // tiles of this cluster
    volatile int* abort = &bars->abort;
    MLA_PROF(long long wacc[kProfSlots] = {0};)
    MLA_PROF(const long long t_kernel0 = clock64();)

    if (threadIdx.x == 0) {
        for (int i = 0; i < 6; ++i) {
            mbar_init(&bars->full[i], 1);
            mbar_init(&bars->stg_empty[i], kConvThreads);
            mbar_init(&bars->bf_full[i], kConvThreads);
            mbar_init(&bars->bf_empty[i], 1);
        }
        for (int i = 0; i < kSBufs; ++i) {
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->p_full[i], 256);
            mbar_init(&bars->o_done[i], 1);
        }
        for (int i = 0; i < kSBufs; ++i) mbar_init(&bars->s_read[i], 128);
        for (int i = 0; i < kXBufs; ++i)
            for (int w = 0; w < 4; ++w) {
                mbar_init(&bars->x_full[i][w], 1);
                mbar_init(&bars->x_free[i][w], 1);
            }
        mbar_init(&bars->q_ready, 128);
        // the bytes the peer pushes for tiles 0 and 1 (later tiles are announced by
        // the softmax warp that consumed the buffer's previous tile)
        for (int i = 0; i < kXBufs; ++i)
            for (int w = 0; w < 4; ++w) {
                mbar_arrive_expect_tx(&bars->x_full[i][w], uint32_t(kXB / 4));   // one warp's 32 rows
                mbar_arrive_expect_tx(&bars->x_free[i][w], 4u);   // the signal freeing the buffer for tile i+2
            }
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(&bars->tmem_base, kTmemCols);
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tm_ckv);
        tma_prefetch_desc(&tm_pe);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    cluster_sync();   // the peer's barriers exist before any remote arrive
    const uint32_t tmem = bars->tmem_base;
    pdl_wait();       // the queries (and the cache) may come from the previous kernels
    pdl_trigger();

    // Register split per warpgroup, set at the top of each role. setmaxnreg.inc
    // draws only on registers other warpgroups of this CTA released, so the
    // per-warp sum over the five warpgroups must stay within 5 x the launch
    // count (96): the TMA / MMA warpgroup gives 16 back, the exchange and
    // converter warpgroups 24 each, the softmax warpgroups take 32 more each.
    if (n > 0) {
        if (warp < 4) setmaxnreg_dec<kRegBase>();
        if (warp == 0 && lane == 0) {
            // ------------------------------------------------------------ TMA producer
            TileIter it = locate(p, t_begin);
            for (int64_t i = 0; i < n; ++i, advance(p, it)) {
                const int32_t row = int32_t((it.g / p.sq) * p.sk + it.j * NK);
                trace_put(p, 0, i * 16 + 1);
                if constexpr (Tr::kConvert) {
                    bool okp = true;
                    for (int h = 0; h < NK / kStgRows && okp; ++h) {
                        const int64_t k = int64_t(NK / kStgRows) * i + h;
                        const int st = int(k % Tr::kStages);
                        okp = MLA_TW(1, mbar_wait(&bars->stg_empty[st], uint32_t(((k / Tr::kStages) & 1) ^ 1), abort, p.err,
                                        ERR_TIMEOUT_BASE + 1));
                        if (!okp) break;
                        unsigned char* dst = stg + st * kStgBytes;
                        mbar_arrive_expect_tx(&bars->full[st], uint32_t(kStgBytes));
                        tma_load_2d(dst, &tm_ckv, &bars->full[st], int32_t(rank * kHalf), row + h * kStgRows);
                        tma_load_2d(dst + kStgLatBytes, &tm_pe, &bars->full[st], int32_t(rank * kRopeHalf),
                                    row + h * kStgRows);
                    }
                    if (!okp) break;
                } else {
                    const int sl = int(i % Tr::kSlots);
                    if (!MLA_TW(2, mbar_wait(&bars->bf_empty[sl], uint32_t(((i / Tr::kSlots) & 1) ^ 1), abort, p.err,
                                   ERR_TIMEOUT_BASE + 2)))
                        break;
                    unsigned char* dst = slots + sl * kSlotBytes;
                    mbar_arrive_expect_tx(&bars->full[sl], uint32_t(kSlotBytes));
                    for (int c = 0; c < 4; ++c)
                        tma_load_2d(dst + c * kChunkBytes, &tm_ckv, &bars->full[sl], int32_t(rank * kHalf + c * 64), row);
                    tma_load_2d(dst + 4 * kChunkBytes, &tm_pe, &bars->full[sl], int32_t(rank * kRopeHalf), row);
                }
            }
        } else if (warp == 1 || warp == 2) {
            // ------------------------------------------------------------ MMA issuers
            // Two issuing threads, so neither waits behind the other's instructions:
            // warp 1 issues the score MMAs S(i), warp 2 the P.V MMAs. A thread's
            // commit tracks only its own MMAs, so the order between the two streams
            // is explicit: S(i) writes score buffer i%2 only after P.V(i-2) has
            // completed (o_done), since P(i-2) lives there, and after the exchange
            // warps have read S(i-2) (s_read). P.V(i) is issued only after p_full(i),
            // which follows the completion of S(i); its commit releases the slot.
            constexpr uint32_t idesc_s = instr_desc(Tr::kFmt, 128, NK, 0, 0);
            constexpr uint32_t idesc_o = instr_desc(Tr::kFmt, 128, kHalf, 0, 1);
            const uint32_t smem_slots = smem_u32(slots);
            if (warp == 1 && lane == 0) {
                const uint64_t qd0 = smem_desc(smem_u32(qrope), 16, 512, 4);
                TileIter it = locate(p, t_begin);
                int64_t seg = 0;
                for (int64_t i = 0; i < n; ++i, advance(p, it)) {
                    MLA_TL(9, i);
                    const bool first = (i == 0) || it.j == 0;
                    if (first) {
                        if (!MLA_TW(4, mbar_wait(&bars->q_ready, uint32_t(seg & 1), abort, p.err, ERR_TIMEOUT_BASE + 4))) break;
                        ++seg;
                    }
                    const int sl = int(i % Tr::kSlots);
                    trace_put(p, 1, i * 16 + 1);
                    uint64_t* fb = Tr::kConvert ? &bars->bf_full[sl] : &bars->full[sl];
                    if (!MLA_TW(5, mbar_wait(fb, uint32_t((i / Tr::kSlots) & 1), abort, p.err, ERR_TIMEOUT_BASE + 5))) break;
                    const int sb = int(i % kSBufs);
                    if (i >= kSBufs) {
                        // the exchange warps have read my partial of tile i-2, and P.V(i-2)
                        // has consumed P(i-2), from this buffer
                        const uint32_t par = uint32_t(((i - kSBufs) / kSBufs) & 1);
                        if (!MLA_TW(13, mbar_wait(&bars->s_read[sb], par, abort, p.err, ERR_TIMEOUT_BASE + 13)) ||
                            !MLA_TW(25, mbar_wait(&bars->o_done[sb], par, abort, p.err, ERR_TIMEOUT_BASE + 25)))
                            break;
                    }
                    tc_fence_after();
                    const uint32_t base = smem_slots + sl * kSlotBytes;
                    // B = K [64 keys x 16 dims], K-major: latent chunk k/4 (128B swizzle,
                    // +32 B per k-step), then the rope chunk (64B swizzle, +32 B per
                    // k-step) against the rope query slice in shared memory.
                    MLA_PROF(const long long t_si = clock64();)
                    MLA_TL(8, i);
                    const uint64_t bd0 = smem_desc(base, 16, 1024, 2);
                    const uint64_t rd0 = smem_desc(base + 4 * kChunkBytes, 16, 512, 4);
                    const uint32_t d_s = tmem + kTmemS + sb * NK;
#pragma unroll
                    for (int k = 0; k < kHalf / 16; ++k)
                        mma_ts(d_s, tmem + kTmemQ + k * 8,
                               bd0 + uint64_t(((k >> 2) * kChunkBytes + (k & 3) * 32) >> 4), idesc_s, k > 0 ? 1u : 0u);
#pragma unroll
                    for (int k = 0; k < kRopeHalf / 16; ++k)
                        mma_ss(d_s, qd0 + uint64_t((k * 32) >> 4), rd0 + uint64_t((k * 32) >> 4), idesc_s, 1u);
                    mma_commit(&bars->s_full[sb]);
                    MLA_TL(0, i);
                    MLA_PROF(wacc[16] += clock64() - t_si;)
                    trace_put(p, 1, i * 16 + 2);
                }
            } else if (warp == 2 && lane == 0) {
                // P.V of tile i: O += P(i) . V(i) (M = 128 heads, N = 256 latent dims,
                // K = 64 keys), A = P from TMEM, B = the key tile's latent half,
                // MN-major, 128B swizzle (LBO = stride between 64-dim chunks, SBO =
                // stride between 8-key groups). Releases the slot, signals o_done.
                TileIter it = locate(p, t_begin);
                for (int64_t i = 0; i < n; ++i, advance(p, it)) {
                    const bool first = (i == 0) || it.j == 0;
                    const int sb = int(i % kSBufs);
                    if (!MLA_TW(3, mbar_wait(&bars->p_full[sb], uint32_t((i / kSBufs) & 1), abort, p.err, ERR_TIMEOUT_BASE + 3)))
                        break;
                    tc_fence_after();
                    MLA_TL(6, i);
                    MLA_PROF(const long long t_pv = clock64();)
                    const int sl = int(i % Tr::kSlots);
                    const uint32_t base = smem_slots + sl * kSlotBytes;
                    const uint32_t p_tmem = tmem + kTmemS + sb * NK;
                    const uint64_t vd0 = smem_desc(base, kChunkBytes, 1024, 2);
#pragma unroll
                    for (int k = 0; k < NK / 16; ++k)
                        mma_ts(tmem + kTmemO, p_tmem + k * 8, vd0 + uint64_t((k * 16 * 128) >> 4), idesc_o,
                               (first && k == 0) ? 0u : 1u);
                    if constexpr (kExact) {   // + P_lo . V (P_lo in columns NK/2.. of the buffer)
#pragma unroll
                        for (int k = 0; k < NK / 16; ++k)
                            mma_ts(tmem + kTmemO, p_tmem + NK / 2 + k * 8, vd0 + uint64_t((k * 16 * 128) >> 4),
                                   idesc_o, 1u);
                    }
                    mma_commit(&bars->bf_empty[sl]);
                    mma_commit(&bars->o_done[sb]);
                    MLA_TL(1, i);
                    MLA_PROF(wacc[17] += clock64() - t_pv;)
                }
            }
        } else if (warp >= 8 && warp < 12) {
            setmaxnreg_dec<kRegExchange>();
            // ------------------------------------------------------------ exchange
            // Per tile: loads the next segment's query when one starts (latent slice
            // into TMEM, rope slice into shared memory), waits for my partial scores,
            // and pushes them into the peer's exchange buffer with st.async (bytes
            // counted on the peer's barrier). Exchange buffer b (= tile % 2) of a
            // warp's 32 rows is pushed into only after the peer's matching softmax
            // warp has said (x_free) that it read the buffer's previous tile. Runs
            // ahead of the softmax warps, so the DSMEM transfer is off their path.
            const int row = threadIdx.x - 256;               // head
            const int wq = warp & 3;
            const uint32_t lane_off = uint32_t(wq * 32) << 16;
            const float c = p.c_log2;
            // peer addresses of my exchange row (chunk 0) and of my warp's exchange
            // barriers (buffer 0; buffer b is at +b*kXB / +b*4*8 bytes)
            const uint32_t xpeer0 = map_peer(xbuf + row * 4, peer);
            const uint32_t xbar_peer0 = map_peer(&bars->x_full[0][wq], peer);
            TileIter itp = locate(p, t_begin);
            for (int64_t i = 0; i < n; ++i, advance(p, itp)) {
                MLA_PROF(const long long t_pr = clock64();)
                const bool first = (i == 0) || itp.j == 0;
                const int sb = int(i % kSBufs);
                // A few tiles before this group ends, pull my row of the next group's
                // query into L2, so that loading it at the switch does not wait on
                // DRAM round trips (the switch otherwise costs ~10 tile periods).
                if (itp.j == (itp.tiles > kQPrefetchTiles ? itp.tiles - kQPrefetchTiles : 0) &&
                    i + (itp.tiles - itp.j) < n) {
                    const int64_t gnext = itp.g + 1;
                    const char* qa_n = reinterpret_cast<const char*>(static_cast<const T*>(p.qa) +
                                                                     (gnext * kHeads + row) * kRank + rank * kHalf);
                    const char* qr_n = reinterpret_cast<const char*>(static_cast<const T*>(p.qr) +
                                                                     (gnext * kHeads + row) * kRope + rank * kRopeHalf);
#pragma unroll
                    for (int l = 0; l < int(kHalf * sizeof(T)) / 128; ++l) prefetch_l2(qa_n + l * 128);
                    prefetch_l2(qr_n);
                }
                if (first) {
                    // query of this group: the latent slice into TMEM as bf16/fp16
                    // pairs (32 dims = 16 TMEM columns per step, all 16-byte loads
                    // of a step issued before any conversion), the rope slice into
                    // shared memory (64B-swizzled K-major A operand)
                    __syncwarp();   // tcgen05.st below is warp-collective
                    const int64_t grow = itp.g * kHeads + row;
                    const T* qa = static_cast<const T*>(p.qa) + grow * kRank + rank * kHalf;
                    const T* qr = static_cast<const T*>(p.qr) + grow * kRope + rank * kRopeHalf;
                    constexpr int kV = 16 / sizeof(T);           // elements per 16-byte vector
                    for (int c16 = 0; c16 < kHalf / 32; ++c16) {
                        uint4 v[32 / kV];
#pragma unroll
                        for (int q = 0; q < 32 / kV; ++q)
                            v[q] = __ldg(reinterpret_cast<const uint4*>(qa + c16 * 32) + q);
                        uint32_t r[16];
#pragma unroll
                        for (int q = 0; q < 32 / kV; ++q) {
                            if constexpr (sizeof(T) == 4) {
                                r[2 * q] = pack_bf16(__uint_as_float(v[q].x), __uint_as_float(v[q].y));
                                r[2 * q + 1] = pack_bf16(__uint_as_float(v[q].z), __uint_as_float(v[q].w));
                            } else {                                 // 16-bit storage: already pairs
                                r[4 * q] = v[q].x; r[4 * q + 1] = v[q].y; r[4 * q + 2] = v[q].z; r[4 * q + 3] = v[q].w;
                            }
                        }
                        tmem_st16(tmem + lane_off + kTmemQ + c16 * 16, r);
                    }
                    {
                        uint4 v[kRopeHalf / kV];
#pragma unroll
                        for (int q = 0; q < kRopeHalf / kV; ++q) v[q] = __ldg(reinterpret_cast<const uint4*>(qr) + q);
                        uint32_t r[16];
#pragma unroll
                        for (int q = 0; q < kRopeHalf / kV; ++q) {
                            if constexpr (sizeof(T) == 4) {
                                r[2 * q] = pack_bf16(__uint_as_float(v[q].x), __uint_as_float(v[q].y));
                                r[2 * q + 1] = pack_bf16(__uint_as_float(v[q].z), __uint_as_float(v[q].w));
                            } else {
                                r[4 * q] = v[q].x; r[4 * q + 1] = v[q].y; r[4 * q + 2] = v[q].z; r[4 * q + 3] = v[q].w;
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            *reinterpret_cast<uint4*>(qrope + swz64(uint32_t(row), uint32_t(u))) =
                                make_uint4(r[4 * u], r[4 * u + 1], r[4 * u + 2], r[4 * u + 3]);
                    }
                    tmem_st_wait();
                    fence_proxy_async_smem();   // the rope slice is read by the tensor cores (async proxy)
                    tc_fence_before();
                    mbar_arrive(&bars->q_ready);
                    if (warp == 8 && lane == 0) MLA_TL(10, i);
                }
                // every lane polls, then the warp reconverges: tcgen05.ld is warp-collective
                if (!__all_sync(0xffffffffu, MLA_TW(6, mbar_wait(&bars->s_full[sb], uint32_t((i / kSBufs) & 1), abort, p.err,
                                                       ERR_TIMEOUT_BASE + 6))))
                    break;
                if (warp == 8 && lane == 0) MLA_TL(2, i);
                tc_fence_after();
                const int xb = int(i % kXBufs);
                const int64_t k = i / kXBufs;
                // the peer's buffer xb must no longer hold tile i-2 unread; once it is
                // free, arm the barrier for the signal that frees it for tile i+2
                if (!__all_sync(0xffffffffu, MLA_TW(7, mbar_wait(&bars->x_free[xb][wq], uint32_t((k & 1) ^ 1), abort, p.err,
                                                       ERR_TIMEOUT_BASE + 7, /*cluster_scope=*/true))))
                    break;
                if (lane == 0 && i >= kXBufs && i + kXBufs < n) mbar_arrive_expect_tx(&bars->x_free[xb][wq], 4u);
                // st.async pushes my partial (log2 units in fp16; raw fp32 in the exact
                // variant), counted on the peer's barrier
#pragma unroll
                for (int h = 0; h < NK / 32; ++h) {   // 32 keys at a time
                    uint32_t sr[32];
                    tmem_ld32(tmem + lane_off + kTmemS + sb * NK + h * 32, sr);
                    tmem_ld_wait();
                    if constexpr (kExact) {
#pragma unroll
                        for (int e = 0; e < 8; ++e)    // chunk h*8+e: keys 32h+4e .. +3
                            st_async_v4(xpeer0 + uint32_t(xb) * kXB + uint32_t(h * 8 + e) * (kHeads * 16),
                                        __uint_as_float(sr[4 * e]), __uint_as_float(sr[4 * e + 1]),
                                        __uint_as_float(sr[4 * e + 2]), __uint_as_float(sr[4 * e + 3]),
                                        xbar_peer0 + uint32_t(xb) * uint32_t(4 * 8));
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {  // chunk h*4+e: keys 32h+8e .. +7
                            uint32_t w[4];
#pragma unroll
                            for (int q = 0; q < 4; ++q)
                                w[q] = pack_x16(__uint_as_float(sr[8 * e + 2 * q]), __uint_as_float(sr[8 * e + 2 * q + 1]),
                                                c);
                            st_async_v4(xpeer0 + uint32_t(xb) * kXB + uint32_t(h * 4 + e) * (kHeads * 16),
                                        __uint_as_float(w[0]), __uint_as_float(w[1]), __uint_as_float(w[2]),
                                        __uint_as_float(w[3]), xbar_peer0 + uint32_t(xb) * uint32_t(4 * 8));
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&bars->s_read[sb]);
                if (warp == 8 && lane == 0) MLA_TL(3, i);
                MLA_PROF(wacc[19] += clock64() - t_pr;)
            }
        } else if ((warp >= 4 && warp < 8) || (warp >= 12 && warp < 16)) {
            setmaxnreg_inc<kRegSoftmax>();
            // ------------------------------------------------------------ softmax
            // Two warps per TMEM lane quarter: warps 4-7 take keys 0-31 of every
            // tile, warps 12-15 keys 32-63. Per tile each warp adds my partial scores
            // (TMEM) and the peer's (exchange buffer) for its 32 keys, and the two
            // warps of a quarter swap their row maxima through shared memory (named
            // barrier 1 + quarter), so both hold the same tile maximum, take the same
            // lazy-rescale decision and share one running maximum. Each writes its
            // half of P, keeps its own partial row sum, rescales and stores its 128
            // columns of the O half; the sums are added at the epilogue. After both
            // have read the exchange buffer, the first warp announces the bytes of
            // the buffer's next tile and tells the peer's exchange warp (a 4-byte
            // st.async completing its x_free barrier) that it may push them. Scores are
            // in log2 units here (the exchanged partials are).
            const int wq = warp & 3;
            const int hk = warp >= 12 ? 1 : 0;                // key half
            const int row = wq * 32 + lane;                  // head
            const uint32_t lane_off = uint32_t(wq * 32) << 16;
            const uint32_t bar_id = 1u + uint32_t(wq);
            const float c = p.c_log2;
            const float tau = 8.0f;                          // lazy rescale threshold (log2 units)
            // peer addresses of this quarter's x_free barrier and landing word
            // (buffer 0; buffer b is at +b*4*8 / +b*4*4 bytes)
            const uint32_t xfree_peer0 = map_peer(&bars->x_free[0][wq], peer);
            const uint32_t sink_peer0 = map_peer(&bars->sink[0][wq], peer);
            int64_t seg_local = 0;
            float m_run = -INFINITY, l_run = 0.f;            // l_run: sum over my key half
            TileIter it = locate(p, t_begin);
            for (int64_t i = 0; i < n; ++i) {
                const bool first = (i == 0) || it.j == 0;
                const bool last = (i + 1 == n) || (it.j + 1 == it.tiles);
                const int sb = int(i % kSBufs);
                if (first) {
                    m_run = -INFINITY;
                    l_run = 0.f;
                }
                if (!__all_sync(0xffffffffu, MLA_TW(14, mbar_wait(&bars->s_full[sb], uint32_t((i / kSBufs) & 1), abort,
                                                                  p.err, ERR_TIMEOUT_BASE + 14))))
                    break;
                tc_fence_after();
                const int xb = int(i % kXBufs);
                if (!__all_sync(0xffffffffu, MLA_TW(8, mbar_wait(&bars->x_full[xb][wq], uint32_t((i / kXBufs) & 1), abort,
                                                                 p.err, ERR_TIMEOUT_BASE + 8, /*cluster_scope=*/true))))
                    break;
                if (warp == 4 && lane == 0) MLA_TL(4, i);
                // my partial of my 32 keys (the score buffer is not reused before P.V(i)
                // is issued), rounded as the peer rounded the one it pushed, plus the
                // peer's partial
                MLA_PROF(const long long t_fi = clock64();)
                float s[32];
                {
                    uint32_t sr[32];
                    tmem_ld32(tmem + lane_off + kTmemS + sb * NK + hk * 32, sr);
                    if constexpr (kExact) {
                        // fp32 chunks hk*8+e: the two halves add the same two values in
                        // either order, so both CTAs hold the same sums
                        const float4* xr = reinterpret_cast<const float4*>(
                            reinterpret_cast<const unsigned char*>(xbuf) + xb * kXB + (hk * 8 * kHeads + row) * 16);
                        float4 pv[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) pv[e] = xr[e * kHeads];
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            s[4 * e] = (__uint_as_float(sr[4 * e]) + pv[e].x) * c;
                            s[4 * e + 1] = (__uint_as_float(sr[4 * e + 1]) + pv[e].y) * c;
                            s[4 * e + 2] = (__uint_as_float(sr[4 * e + 2]) + pv[e].z) * c;
                            s[4 * e + 3] = (__uint_as_float(sr[4 * e + 3]) + pv[e].w) * c;
                        }
                    } else {
                        const uint4* xr = reinterpret_cast<const uint4*>(
                            reinterpret_cast<const unsigned char*>(xbuf) + xb * kXB + (hk * 4 * kHeads + row) * 16);
                        uint4 pv[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) pv[e] = xr[e * kHeads];
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const uint32_t pw[4] = {pv[e].x, pv[e].y, pv[e].z, pv[e].w};
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int k = 8 * e + 2 * q;
                                const float2 mine =
                                    unpack_x16(pack_x16(__uint_as_float(sr[k]), __uint_as_float(sr[k + 1]), c));
                                const float2 peer = unpack_x16(pw[q]);
                                s[k] = mine.x + peer.x;
                                s[k + 1] = mine.y + peer.y;
                            }
                        }
                    }
                }
                MLA_PROF(wacc[20] += clock64() - t_fi; const long long t_f1 = clock64();)
                const int64_t key0 = it.j * NK + hk * 32;
                if (key0 + 32 > it.keys) {            // ragged last tile of a group (warp-uniform)
                    const int valid = int(it.keys - key0);
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (e >= valid) s[e] = -INFINITY;
                }
                float m4[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) m4[q] = fmaxf(fmaxf(s[q], s[q + 4]), fmaxf(s[q + 8], s[q + 12]));
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    m4[q] = fmaxf(m4[q], fmaxf(fmaxf(s[q + 16], s[q + 20]), fmaxf(s[q + 24], s[q + 28])));
                const float mh = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
                // swap half maxima with the other warp of this quarter (double-buffered
                // by tile parity: my next write follows the next barrier, which the
                // other warp reaches only after reading this one)
                float* xm = reinterpret_cast<float*>(bars->xmax[i & 1]);
                xm[hk * kHeads + row] = mh;
                named_bar_sync(bar_id, 64);
                float mt = fmaxf(mh, xm[(hk ^ 1) * kHeads + row]);
                // Both warps have read the exchange buffer (each passed the barrier after
                // a maximum that depends on every value it read): announce the bytes of
                // the buffer's next tile (i+2) and free it for the peer's push.
                if (hk == 0 && lane == 0) {
                    if (i + kXBufs < n) mbar_arrive_expect_tx(&bars->x_full[xb][wq], uint32_t(kXB / 4));
                    st_async_b32(sink_peer0 + uint32_t(xb) * 16u, mt, xfree_peer0 + uint32_t(xb) * 32u);
                }
                if (first) {
                    m_run = mt;
                } else if (__any_sync(0xffffffffu, mt > m_run + tau)) {
                    // Lazy rescale, decided per quarter (both warps see the same maxima;
                    // the peer CTA sees the same scores, so it decides the same): every
                    // row moves to its new maximum (alpha <= 1). Waits for P.V of the
                    // previous tile first; each warp rescales its 128 O columns.
                    const int pb = int((i - 1) % kSBufs);
                    if (!__all_sync(0xffffffffu, MLA_TW(9, mbar_wait(&bars->o_done[pb], uint32_t(((i - 1) / kSBufs) & 1),
                                                                     abort, p.err, ERR_TIMEOUT_BASE + 9))))
                        break;
                    tc_fence_after();
                    mt = fmaxf(mt, m_run);
                    const float alpha = ex2(m_run - mt);
#pragma unroll 1
                    for (int c32 = 0; c32 < kHalf / 64; ++c32) {
                        uint32_t o[32];
                        const uint32_t col = kTmemO + hk * (kHalf / 2) + c32 * 32;
                        tmem_ld32(tmem + lane_off + col, o);
                        tmem_ld_wait();
                        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st32(tmem + lane_off + col, o);
                    }
                    tmem_st_wait();
                    l_run *= alpha;
                    m_run = mt;
                }
                MLA_PROF(wacc[21] += clock64() - t_f1; const long long t_f2 = clock64();)
                const float mc = m_run;
                uint32_t pk[16];                  // P (16-bit pairs); the exact variant's P_hi
                uint32_t pl[kExact ? 16 : 1];     // the exact variant's P_lo = P - P_hi
                float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float p0 = ex2(s[e] - mc);
                    const float p1 = ex2(s[e + 1] - mc);
                    ls[(e >> 1) & 3] += p0 + p1;
                    if constexpr (Tr::kFmt == 0) {
                        __half2 h2 = __floats2half2_rn(p0, p1);
                        pk[e / 2] = *reinterpret_cast<uint32_t*>(&h2);
                        if constexpr (kExact) {
                            const float2 f = __half22float2(h2);
                            __half2 l2 = __floats2half2_rn(p0 - f.x, p1 - f.y);
                            pl[e / 2] = *reinterpret_cast<uint32_t*>(&l2);
                        }
                    } else {
                        pk[e / 2] = pack_bf16(p0, p1);
                        if constexpr (kExact)
                            pl[e / 2] = pack_bf16(p0 - __uint_as_float(pk[e / 2] << 16),
                                                  p1 - __uint_as_float(pk[e / 2] & 0xffff0000u));
                    }
                }
                l_run += (ls[0] + ls[1]) + (ls[2] + ls[3]);
                MLA_PROF(wacc[22] += clock64() - t_f2; const long long t_f3 = clock64();)
                // P overwrites my partial scores of tile i: my exchange warps must have
                // read them first (this warp may be ahead of them, since it needs only
                // the peer's push)
                if (!__all_sync(0xffffffffu, MLA_TW(24, mbar_wait(&bars->s_read[sb], uint32_t((i / kSBufs) & 1), abort,
                                                                  p.err, ERR_TIMEOUT_BASE + 24))))
                    break;
                __syncwarp();
                tmem_st16(tmem + lane_off + kTmemS + sb * NK + hk * 16, pk);
                if constexpr (kExact) tmem_st16(tmem + lane_off + kTmemS + sb * NK + NK / 2 + hk * 16, pl);
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&bars->p_full[sb]);
                if (warp == 4 && lane == 0) MLA_TL(5, i);
                MLA_PROF(wacc[23] += clock64() - t_f3;)
                MLA_PROF(wacc[18] += clock64() - t_fi;)
                if (lane == 0 && warp == 4) trace_put(p, 2, i * 16 + 4);
                if (last) {
                    if (!__all_sync(0xffffffffu, MLA_TW(10, mbar_wait(&bars->o_done[sb], uint32_t((i / kSBufs) & 1), abort,
                                                                      p.err, ERR_TIMEOUT_BASE + 10))))
                        break;
                    tc_fence_after();
                    const int64_t slot = cl * p.max_segs + seg_local;
                    // chunk-major partial output: the 4 dims of chunk ch (dims 4ch..4ch+3) of
                    // head `row` at float4 index ch*128 + row of the slot, so that a warp's 32
                    // rows store 512 contiguous bytes per instruction (a row-per-thread layout
                    // put 32 cache lines into every store and slowed the next group's query
                    // loads at a segment switch)
                    float4* dst = reinterpret_cast<float4*>(p.O_part) + slot * (kRank / 4) * kHeads + row;
                    const int ch0 = (rank * kHalf + hk * (kHalf / 2)) / 4;
#pragma unroll 1
                    for (int c32 = 0; c32 < kHalf / 64; ++c32) {
                        uint32_t o[32];
                        tmem_ld32(tmem + lane_off + kTmemO + hk * (kHalf / 2) + c32 * 32, o);
                        tmem_ld_wait();
                        for (int e = 0; e < 8; ++e)
                            dst[(ch0 + c32 * 8 + e) * kHeads] =
                                make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                                            __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
                    }
                    // the row sum is the sum of the two halves' sums
                    bars->xl[hk * kHeads + row] = l_run;
                    named_bar_sync(bar_id, 64);
                    if (rank == 0 && hk == 0) {
                        p.ml[(slot * kHeads + row) * 2] = m_run;
                        p.ml[(slot * kHeads + row) * 2 + 1] = l_run + bars->xl[kHeads + row];
                    }
                    tc_fence_before();
                    ++seg_local;
                    if (warp == 4 && lane == 0) MLA_TL(11, i);
                }
                advance(p, it);
            }
        } else if (warp >= 16) {
            setmaxnreg_dec<kRegConvert>();
          if constexpr (Tr::kConvert) {
            // ------------------------------------------------------------ fp32 -> bf16
            // Converts four fp32 quarter-tile staging buffers into one bf16 slot.
            // Every thread reads its share of a quarter tile into registers and
            // releases the staging buffer before writing, so the next TMA load can
            // start at once.
            const int ct = (warp - 16) * 32 + lane;
            // Lanes take consecutive 16-byte (4 x fp32) pieces of a staging row, so a
            // warp's shared-memory reads are dense; each piece becomes 8 bytes of bf16.
            constexpr int kU = kStgRows * (kHalf / 4) / kConvThreads;       // latent float4 pieces per thread
            constexpr int kP = kStgRows * (kRopeHalf / 4) / kConvThreads;   // rope float4 pieces per thread
            static_assert(kU * kConvThreads == kStgRows * (kHalf / 4) &&
                          kP * kConvThreads == kStgRows * (kRopeHalf / 4), "converter mapping");
            bool okc = true;
            for (int64_t i = 0; okc && i < n; ++i) {
                const int sl = int(i % Tr::kSlots);
                if (!MLA_TW(11, mbar_wait(&bars->bf_empty[sl], uint32_t(((i / Tr::kSlots) & 1) ^ 1), abort, p.err,
                               ERR_TIMEOUT_BASE + 11)))
                    break;
                if (ct == 0) trace_put(p, 3, i * 16 + 2);
                unsigned char* buf = slots + sl * kSlotBytes;
                for (int h = 0; h < NK / kStgRows; ++h) {
                    const int64_t k = int64_t(NK / kStgRows) * i + h;
                    const int st = int(k % Tr::kStages);
                    if (!MLA_TW(12, mbar_wait(&bars->full[st], uint32_t((k / Tr::kStages) & 1), abort, p.err,
                                   ERR_TIMEOUT_BASE + 12))) {
                        okc = false;
                        break;
                    }
                    MLA_PROF(const long long t_cv = clock64();)
                    const float4* src = reinterpret_cast<const float4*>(stg + st * kStgBytes);
                    float4 a[kU], b[kP];
                    // all loads of the quarter tile first, then the conversions
#pragma unroll
                    for (int q = 0; q < kU; ++q) a[q] = src[ct + q * kConvThreads];
#pragma unroll
                    for (int q = 0; q < kP; ++q) b[q] = src[kStgLatBytes / 16 + ct + q * kConvThreads];
                    // convert and store into the slot, then release the staging buffer:
                    // the stores consume every value read from staging, and a warp issues
                    // in order, so the release cannot issue before all reads returned and
                    // the next TMA write into the buffer cannot overtake them
#pragma unroll
                    for (int q = 0; q < kU; ++q) {
                        const int f = ct + q * kConvThreads;          // float4 index in the quarter tile
                        const int r = h * kStgRows + (f >> 6), c4 = f & 63;
                        *reinterpret_cast<uint2*>(buf + (c4 >> 4) * kChunkBytes +
                                                  swz128(uint32_t(r), uint32_t((c4 & 15) >> 1)) + (c4 & 1) * 8) =
                            make_uint2(pack_bf16(a[q].x, a[q].y), pack_bf16(a[q].z, a[q].w));
                    }
#pragma unroll
                    for (int q = 0; q < kP; ++q) {
                        const int f = ct + q * kConvThreads;
                        const int r = h * kStgRows + (f >> 3), c4 = f & 7;
                        *reinterpret_cast<uint2*>(buf + 4 * kChunkBytes + swz64(uint32_t(r), uint32_t(c4 >> 1)) +
                                                  (c4 & 1) * 8) =
                            make_uint2(pack_bf16(b[q].x, b[q].y), pack_bf16(b[q].z, b[q].w));
                    }
                    mbar_arrive(&bars->stg_empty[st]);
                    MLA_PROF(wacc[15] += clock64() - t_cv;)
                }
                if (!okc) break;
                fence_proxy_async_smem();
                mbar_arrive(&bars->bf_full[sl]);
                if (warp == 16 && lane == 0) MLA_TL(7, i);
            }
          }
        }
    }

#ifdef MLA_TC_PROFILE
    if (p.prof && lane == 0 && (warp == 0 || warp == 1 || warp == 16 || warp == 4 || warp == 8)) {   // one per role
        for (int k = 0; k < kProfSlots; ++k)
            if (wacc[k]) atomicAdd(reinterpret_cast<unsigned long long*>(p.prof + blockIdx.x * kProfSlots + k),
                                   (unsigned long long)wacc[k]);
        if (warp == 0)
            atomicAdd(reinterpret_cast<unsigned long long*>(p.prof + blockIdx.x * kProfSlots + 0),
                      (unsigned long long)(clock64() - t_kernel0));
    }
#endif
    if (threadIdx.x == 0) trace_put(p, 4, 1);
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) trace_put(p, 5, bars->abort ? 2 : 1);
    if (bars->abort) {
        // let in-flight asynchronous copies and MMAs drain before freeing resources
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 2000000ull) { }
    }
    tc_fence_after();
    __syncwarp();
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
    __syncwarp();
    cluster_sync();
    if (threadIdx.x == 0) trace_put(p, 6, 1);
    if (p.trace) __threadfence_system();
}

// Combine the segments of every (group, head) row into a normalised context.
// One CTA per (group, piece of P dims), one thread per head: each reads its
// row's piece from every segment of the group (the cluster segments covering a
// group are contiguous), chunk-major so that a warp's reads are contiguous, and
// the result goes out through shared memory so that rows are written
// contiguously. P (32 down to 4) is chosen by the host so that few groups (long
// contexts, small batches) still spread over every SM.
template <typename OutT, int kCombinePiece>
__global__ void __launch_bounds__(kHeads) combine_kernel(const Params p, OutT* __restrict__ O_norm, int64_t groups,
                                                         float* __restrict__ lse)
{
    pdl_wait();
    pdl_trigger();
    __shared__ float tile[kHeads][kCombinePiece + 1];
    constexpr int kPieces = kRank / kCombinePiece;
    const int64_t g = blockIdx.x / kPieces;
    const int piece = int(blockIdx.x % kPieces);
    const int h = threadIdx.x;
    if (g >= groups) return;
    const int64_t b = g / p.sq, qg = g % p.sq;
    const int64_t t0 = b * tiles_before(p, p.sq) + tiles_before(p, qg);   // first global tile of g
    const int64_t t1 = t0 + group_tiles(p, g);                            // exclusive
    const int64_t c0 = t0 / p.tiles_per_cluster, c1 = (t1 - 1) / p.tiles_per_cluster;
    // online merge over the segments, four at a time so that their loads are in
    // flight together (a long context spreads one group over many clusters)
    float M = -INFINITY, L = 0.f;
    float acc[kCombinePiece];
#pragma unroll
    for (int e = 0; e < kCombinePiece; ++e) acc[e] = 0.f;
    for (int64_t c = c0; c <= c1; c += 4) {
        float m[4], l[4];
        float4 v[4][kCombinePiece / 4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (c + u > c1) { m[u] = -INFINITY; l[u] = 0.f; continue; }
            const int64_t slot = (c + u) * p.max_segs + (g - locate(p, (c + u) * p.tiles_per_cluster).g);
            m[u] = p.ml[(slot * kHeads + h) * 2];
            l[u] = p.ml[(slot * kHeads + h) * 2 + 1];
            const float4* src = reinterpret_cast<const float4*>(p.O_part) + slot * (kRank / 4) * kHeads +
                                int64_t(piece * (kCombinePiece / 4)) * kHeads + h;
#pragma unroll
            for (int e = 0; e < kCombinePiece / 4; ++e) v[u][e] = src[e * kHeads];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (c + u > c1) break;
            const float Mn = fmaxf(M, m[u]);     // finite: a segment has at least one key
            const float sc = exp2f(M - Mn), w = exp2f(m[u] - Mn);
            L = L * sc + w * l[u];
#pragma unroll
            for (int e = 0; e < kCombinePiece / 4; ++e) {
                acc[4 * e] = acc[4 * e] * sc + w * v[u][e].x;
                acc[4 * e + 1] = acc[4 * e + 1] * sc + w * v[u][e].y;
                acc[4 * e + 2] = acc[4 * e + 2] * sc + w * v[u][e].z;
                acc[4 * e + 3] = acc[4 * e + 3] * sc + w * v[u][e].w;
            }
            M = Mn;
        }
    }
    const float inv = 1.f / L;
    // log-sum-exp of the row's scaled scores (M and log2(L) are in log2 units)
    if (lse && piece == 0) lse[g * kHeads + h] = (M + log2f(L)) * 0.69314718055994531f;
#pragma unroll
    for (int e = 0; e < kCombinePiece; ++e) tile[h][e] = acc[e] * inv;
    __syncthreads();
    OutT* dst = O_norm + g * kHeads * kRank + piece * kCombinePiece;
#pragma unroll 4
    for (int k = 0; k < kCombinePiece; ++k) {   // 128 consecutive elements: 4 rows x 32 dims
        const int idx = k * kHeads + h;
        const int r = idx / kCombinePiece, col = idx % kCombinePiece;
        dst[int64_t(r) * kRank + col] = cvt<OutT>(tile[r][col]);
    }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

// 2-D map over a row-major [rows, cols] array; swizzle 0 (none), 64 or 128 bytes.
template <typename T>
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, uint32_t box_cols, uint32_t box_rows,
              int swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    const CUtensorMapDataType dt = std::is_same<T, float>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                  : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(cols) * sizeof(T)};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : swizzle == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

struct Plan {
    int64_t groups, total_tiles, tiles_per_cluster, nclusters;
    int max_segs;
    size_t off_O, off_ml, off_norm, total;
};

int64_t tiles_of(const AArgs& a, int64_t q) {
    const int64_t k = a.causal ? a.sk - a.sq + q + 1 : a.sk;
    return (k + NK - 1) / NK;
}

Plan make_plan(const AArgs& a) {
    Plan pl{};
    pl.groups = a.batch * a.sq;
    int64_t per_batch = 0, min_tiles = INT64_MAX;
    for (int64_t q = 0; q < a.sq; ++q) {
        const int64_t n = tiles_of(a, q);
        per_batch += n;
        min_tiles = n < min_tiles ? n : min_tiles;
    }
    pl.total_tiles = per_batch * a.batch;
    int64_t ncl = sm_count() / 2;
    if (const char* e = getenv("MLA_TC_MAX_CLUSTERS")) {   // debug knob
        const int64_t lim = atoll(e);
        if (lim > 0 && lim < ncl) ncl = lim;
    }
    if (ncl < 1) ncl = 1;
    if (ncl > pl.total_tiles) ncl = pl.total_tiles;
    pl.tiles_per_cluster = (pl.total_tiles + ncl - 1) / ncl;
    pl.nclusters = (pl.total_tiles + pl.tiles_per_cluster - 1) / pl.tiles_per_cluster;
    pl.max_segs = int((pl.tiles_per_cluster + min_tiles - 1) / min_tiles + 1);
    const int64_t slots = pl.nclusters * pl.max_segs;
    size_t off = 0;
    pl.off_O = off;    off = align_up(off + size_t(slots) * kHeads * kRank * 4, 256);
    pl.off_ml = off;   off = align_up(off + size_t(slots) * kHeads * 2 * 4, 256);
    pl.off_norm = off; off = align_up(off + size_t(pl.groups) * kHeads * kRank * 4, 256);
    pl.total = off;
    return pl;
}

}  // namespace tc

bool tc_attention_supported(const AArgs& a) {
    return a.heads == tc::kHeads && a.kv_rank == tc::kRank && a.rope == tc::kRope && a.sk > 0 &&
           a.batch * a.sk < (int64_t(1) << 31);
}

template <typename T>
size_t tc_attention_workspace(const AArgs& a) {
    if constexpr (std::is_same<T, double>::value) return 0;
    else return tc::make_plan(a).total;
}

template <typename T>
mla_status_t tc_attention(const AArgs& a, cudaStream_t st, bool exact) {
    if constexpr (std::is_same<T, double>::value) {
        return set_error(MLA_ERR_UNSUPPORTED, "MLA: tensor-core attention has no fp64 variant");
    } else {
        using namespace tc;
        const Plan pl = make_plan(a);
        char* ws = static_cast<char*>(a.workspace);
        Params p{};
        p.qa = a.q_absorbed;
        p.qr = a.q_rope;
        p.O_part = reinterpret_cast<float*>(ws + pl.off_O);
        p.ml = reinterpret_cast<float*>(ws + pl.off_ml);
        DeviceStatus* dst = nullptr;
        MLA_TRY(device_status_block(&dst));
        p.err = &dst->code;
        p.batch = a.batch; p.sq = a.sq; p.sk = a.sk; p.causal = a.causal;
        p.c_log2 = float(1.4426950408889634 / a.scale);
        p.total_tiles = pl.total_tiles;
        p.tiles_per_cluster = pl.tiles_per_cluster;
        p.max_segs = pl.max_segs;
        float* O_norm = reinterpret_cast<float*>(ws + pl.off_norm);

        // fp32 storage: unswizzled quarter-tile boxes into staging (latent half, rope
        // half); 16-bit storage: straight into the slots, 64-dim latent chunks with
        // the 128-byte swizzle and the 32-dim rope half with the 64-byte swizzle
        CUtensorMap tm_ckv, tm_pe;
        const bool direct = !Traits<T>::kConvert;
        const int64_t rows = a.batch * a.sk;
        const uint32_t box_rows = direct ? uint32_t(NK) : uint32_t(kStgRows);
        if (!make_map<T>(&tm_ckv, a.c_kv, rows, kRank, direct ? 64 : kHalf, box_rows, direct ? 128 : 0) ||
            !make_map<T>(&tm_pe, a.pe_cache, rows, kRope, kRopeHalf, box_rows, direct ? 64 : 0))
            return set_error(MLA_ERR_CUDA, "MLA: cuTensorMapEncodeTiled failed (alignment of c_kv / pe_cache?)");

        constexpr bool k16 = !std::is_same<T, float>::value;
        if (exact && !k16) return set_error(MLA_ERR_UNSUPPORTED, "MLA: the exact tensor-core attention is for 16-bit storage");
        auto kern = (k16 && exact) ? mla_decode_tc_kernel<T, k16> : mla_decode_tc_kernel<T, false>;
        cudaFuncAttributes fa{};
        if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs != kLaunchRegs ||
            fa.maxThreadsPerBlock < kThreads)
            return set_error(MLA_ERR_CUDA,
                             "MLA: decode kernel compiled with %d registers per thread (expected %d; max threads %d): "
                             "its register split would not fit, not launching", fa.numRegs, kLaunchRegs,
                             fa.maxThreadsPerBlock);
        const size_t smem = (k16 && exact) ? smem_bytes<T, k16>() : smem_bytes<T, false>();
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned(2 * pl.nclusters), 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        int* trace_host = nullptr;
        const size_t trace_bytes = size_t(2 * pl.nclusters) * 32 * sizeof(int);   // 32 words per CTA
        if (getenv("MLA_TC_TRACE")) {   // debug: progress words polled from the host while the kernel runs
            if (cudaHostAlloc(reinterpret_cast<void**>(&trace_host), trace_bytes, cudaHostAllocMapped) == cudaSuccess) {
                memset(trace_host, 0xff, trace_bytes);
                cudaHostGetDevicePointer(reinterpret_cast<void**>(&p.trace), trace_host, 0);
            }
        }
#ifdef MLA_TC_PROFILE
        long long* prof_dev = nullptr;
        const size_t prof_bytes = size_t(2 * pl.nclusters) * kProfSlots * sizeof(long long);
        if (getenv("MLA_TC_PROF") && cudaMalloc(&prof_dev, prof_bytes) == cudaSuccess) {
            cudaMemsetAsync(prof_dev, 0, prof_bytes, st);
            p.prof = prof_dev;
        }
#endif
#ifdef MLA_TC_TIMELINE
        long long* tl_dev = nullptr;
        const size_t tl_bytes = size_t(2) * kTlEvents * kTlTiles * sizeof(long long);
        if (getenv("MLA_TC_TL") && cudaMalloc(&tl_dev, tl_bytes) == cudaSuccess) {
            cudaMemsetAsync(tl_dev, 0, tl_bytes, st);
            p.tl = tl_dev;
        }
#endif
        timing_mark(st, true);
        const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, tm_ckv, tm_pe, p);
        timing_mark(st, false);
#ifdef MLA_TC_TIMELINE
        if (tl_dev) {
            std::vector<long long> h(size_t(2) * kTlEvents * kTlTiles);
            if (cudaMemcpyAsync(h.data(), tl_dev, tl_bytes, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
                cudaStreamSynchronize(st) == cudaSuccess) {
                const int64_t nt = std::min<int64_t>(pl.tiles_per_cluster, kTlTiles);
                for (int c = 0; c < 2; ++c) {
                    auto at = [&](int ev, int64_t i) { return double(h[(c * kTlEvents + ev) * kTlTiles + i]); };
                    double d[10] = {0};
                    int cnt = 0;
                    double e[4] = {0, 0, 0, 0};
                    for (int64_t i = 8; i + 3 < nt - 4; ++i, ++cnt) {
                        e[2] += at(9, i + 2) - at(1, i);        // PV(i) issued -> next iteration starts
                        e[3] += at(3, i) - at(1, i);            // exchange released S(i), relative to PV(i) issued
                        e[0] += at(8, i + 2) - at(9, i + 2);    // iteration start -> S(i+2) issue starts (waits)
                        e[1] += at(0, i + 2) - at(8, i + 2);    // S(i+2) issue (18 MMAs + commit)
                        d[0] += at(5, i + 1) - at(5, i);        // tile period (softmax p_full)
                        d[1] += at(5, i) - at(4, i);            // softmax: x_full seen -> p_full
                        d[2] += at(6, i) - at(5, i);            // p_full -> MMA sees it
                        d[3] += at(1, i) - at(6, i);            // PV issue
                        d[4] += at(0, i + 2) - at(1, i);        // PV(i) issued -> S(i+2) issued
                        d[5] += at(2, i + 2) - at(0, i + 2);    // S(i+2) issued -> exchange sees s_full
                        d[6] += at(3, i + 2) - at(2, i + 2);    // exchange push
                        d[7] += at(4, i + 2) - at(3, i + 2);    // my push done -> softmax sees peer's push
                        d[8] += at(0, i + 2) - at(7, i + 2);    // slot ready -> S issued
                        d[9] += at(4, i) - at(5, i - 1);        // softmax idle between tiles
                    }
                    static const char* nm[10] = {"tile period", "softmax x_full->p_full", "p_full->MMA sees",
                                                 "PV issue", "PV(i)->S(i+2) issued", "S issued->exch s_full",
                                                 "exch push", "push->peer data seen", "slot ready->S issued",
                                                 "softmax idle between tiles"};
                    fprintf(stderr, "[mla timeline] CTA %d, %d tiles: average cycles\n", c, cnt);
                    for (int k = 0; k < 10; ++k) fprintf(stderr, "  %-28s %9.0f\n", nm[k], cnt ? d[k] / cnt : 0.0);
                    {   // the largest gap between consecutive tiles (group switches show here)
                        double mx = 0; int64_t at_i = 0;
                        for (int64_t i = 1; i + 1 < nt; ++i)
                            if (at(4, i + 1) - at(4, i) > mx) { mx = at(4, i + 1) - at(4, i); at_i = i; }
                        fprintf(stderr, "  largest tile gap %.0f cycles after tile %lld\n", mx, (long long)at_i);
                        const int64_t i = at_i;
                        const double z = at(4, i);
                        fprintf(stderr, "  switch (cycles from softmax(i) start): p_full(i) %.0f, epilogue done %.0f, "
                                "push(i) done %.0f, q_ready(i+1) %.0f, S(i+1) issue start %.0f, S(i+1) issued %.0f, "
                                "exch s_full(i+1) %.0f, push(i+1) done %.0f, softmax(i+1) start %.0f\n",
                                at(5, i) - z, at(11, i) - z, at(3, i) - z, at(10, i + 1) - z, at(8, i + 1) - z,
                                at(0, i + 1) - z, at(2, i + 1) - z, at(3, i + 1) - z, at(4, i + 1) - z);
                    }
                    fprintf(stderr, "  %-28s %9.0f\n  %-28s %9.0f\n  %-28s %9.0f\n  %-28s %9.0f\n",
                            "  of which loop step", cnt ? e[2] / cnt : 0.0, "  of which waits", cnt ? e[0] / cnt : 0.0,
                            "  of which S issue", cnt ? e[1] / cnt : 0.0, "s_read(i) - PV(i) issued", cnt ? e[3] / cnt : 0.0);
                }
            }
            cudaFree(tl_dev);
        }
#endif
#ifdef MLA_TC_PROFILE
        if (prof_dev) {
            static const char* names[kProfSlots] = {
                "kernel total", "prod stg/slot empty", "prod slot empty(16b)", "mma p_full", "mma q_ready",
                "mma slot ready", "soft s_full", "soft x_free", "soft x_full", "soft o_done(rescale)",
                "soft o_done(epilogue)", "conv bf_empty", "conv stage full", "mma s_read", "soft s_full", "conv work", "mma S issue",
                "mma PV issue", "soft finish work", "exch total", " fin: ld+add", " fin: max+resc",
                " fin: exp+pack", " fin: P store", "soft s_read", ""};
            const int64_t nb = 2 * pl.nclusters;
            long long* h = static_cast<long long*>(malloc(prof_bytes));
            if (h && cudaMemcpyAsync(h, prof_dev, prof_bytes, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
                cudaStreamSynchronize(st) == cudaSuccess) {
                fprintf(stderr, "[mla prof] per-CTA average kcycles over %lld CTAs, %lld tiles per cluster\n",
                        (long long)nb, (long long)pl.tiles_per_cluster);
                for (int k = 0; k < kProfSlots; ++k) {
                    if (!names[k][0]) continue;
                    double sum = 0;
                    for (int64_t b = 0; b < nb; ++b) sum += double(h[b * kProfSlots + k]);
                    fprintf(stderr, "  %-24s %10.1f\n", names[k], sum / nb / 1000.0);
                }
            }
            free(h);
            cudaFree(prof_dev);
        }
#endif
        if (le != cudaSuccess) {
            cudaGetLastError();
            return set_error(MLA_ERR_CUDA, "MLA: launch of the tensor-core attention kernel failed: %s",
                             cudaGetErrorString(le));
        }
        MLA_TRY(check_launch("tensor-core attention"));
        if (trace_host) {
            cudaEvent_t ev;
            cudaEventCreate(&ev);
            cudaEventRecord(ev, st);
            for (int k = 0; k < 100 && cudaEventQuery(ev) == cudaErrorNotReady; ++k) usleep(50000);
            const bool done = cudaEventQuery(ev) == cudaSuccess;
            fprintf(stderr, "[mla trace] kernel %s; grid %lld CTAs\n", done ? "finished" : "STILL RUNNING after 5 s",
                    (long long)(2 * pl.nclusters));
            for (int64_t b = 0; b < 2 * pl.nclusters; ++b) {
                const volatile int* t = trace_host + b * 32;
                fprintf(stderr, "  cta %3lld producer %d mma %d softmax %d converter %d end %d sync %d exit %d\n",
                        (long long)b, t[0], t[1], t[2], t[3], t[4], t[5], t[6]);
            }
            // a kernel still running may write the buffer: keep it mapped (leaked) in that case
            if (!done) return set_error(MLA_ERR_CUDA, "MLA: tensor-core attention did not finish (trace printed)");
            cudaFreeHost(trace_host);
        }
        // combine piece width: the widest of 32 / 16 / 8 / 4 dims that gives two CTAs per SM
        int piece = 32;
        while (piece > 4 && pl.groups * (kRank / piece) < 2 * int64_t(sm_count())) piece /= 2;
        if (const char* e = getenv("MLA_COMBINE_PIECE")) {   // debug / tuning knob: 32, 16, 8 or 4
            const int v = atoi(e);
            if (v == 32 || v == 16 || v == 8 || v == 4) piece = v;
        }
        const unsigned cblocks = unsigned(pl.groups * (kRank / piece));
        auto combine = [&](auto out_tag, void* out) -> mla_status_t {
            using OutT = decltype(out_tag);
            OutT* o = static_cast<OutT*>(out);
            const int64_t gs = pl.groups;
            if (piece == 32) launch_pdl(combine_kernel<OutT, 32>, dim3(cblocks), dim3(kHeads), 0, st, p, o, gs, a.lse);
            else if (piece == 16) launch_pdl(combine_kernel<OutT, 16>, dim3(cblocks), dim3(kHeads), 0, st, p, o, gs, a.lse);
            else if (piece == 8) launch_pdl(combine_kernel<OutT, 8>, dim3(cblocks), dim3(kHeads), 0, st, p, o, gs, a.lse);
            else launch_pdl(combine_kernel<OutT, 4>, dim3(cblocks), dim3(kHeads), 0, st, p, o, gs, a.lse);
            return check_launch("segment combine");
        };
        if (a.v_dim % 32 != 0) {   // W_uv projection on CUDA cores from an fp32 context
            MLA_TRY(combine(float{}, O_norm));
            return attn_out_normalized<T>(a, O_norm, st);
        }
        if constexpr (std::is_same<T, float>::value) {
            if (a.W_uv_bf16) {   // pre-packed W_uv: bf16 context, kind::f16 projection, fp32 output
                __nv_bfloat16* ctx16 = reinterpret_cast<__nv_bfloat16*>(O_norm);
                MLA_TRY(combine(__nv_bfloat16{}, ctx16));
                TcGemm g{};
                g.A = ctx16; g.a_dims[0] = kRank; g.a_dims[1] = kHeads; g.a_dims[2] = pl.groups;
                g.a_ld[0] = kRank; g.a_ld[1] = int64_t(kHeads) * kRank;
                g.B = a.W_uv_bf16; g.b_mn = false; g.b_dims[0] = kRank; g.b_dims[1] = a.v_dim; g.b_dims[2] = kHeads;
                g.b_ld[0] = kRank; g.b_ld[1] = a.v_dim * kRank;
                g.M = pl.groups; g.N = a.v_dim; g.K = kRank; g.Z = kHeads; g.spb = 1; g.k_chunk = kRank;
                g.C = a.out; g.c_is_t = false; g.c_ldm = int64_t(kHeads) * a.v_dim; g.c_ldz = a.v_dim;
                g.bn = a.v_dim % 256 == 0 ? 256 : 128; g.err = p.err;
                return tc_gemm<__nv_bfloat16>(g, st);
            }
        }
        // context in the storage dtype, then out[:, h] = ctx[:, h] @ W_uv[h]^T on the tensor cores
        T* ctx = reinterpret_cast<T*>(O_norm);
        MLA_TRY(combine(T{}, ctx));
        TcGemm g{};
        g.A = ctx; g.a_dims[0] = kRank; g.a_dims[1] = kHeads; g.a_dims[2] = pl.groups;
        g.a_ld[0] = kRank; g.a_ld[1] = int64_t(kHeads) * kRank;
        g.B = a.W_uv; g.b_mn = false; g.b_dims[0] = kRank; g.b_dims[1] = a.v_dim; g.b_dims[2] = kHeads;
        g.b_ld[0] = kRank; g.b_ld[1] = a.v_dim * kRank;
        g.M = pl.groups; g.N = a.v_dim; g.K = kRank; g.Z = kHeads; g.spb = 1; g.k_chunk = kRank;
        g.C = a.out; g.c_is_t = true; g.c_ldm = int64_t(kHeads) * a.v_dim; g.c_ldz = a.v_dim;
        g.bn = a.v_dim % 256 == 0 ? 256 : 128; g.err = p.err;
        return tc_gemm<T>(g, st);
    }
}

template size_t tc_attention_workspace<float>(const AArgs&);
template size_t tc_attention_workspace<double>(const AArgs&);
template size_t tc_attention_workspace<__half>(const AArgs&);
template size_t tc_attention_workspace<__nv_bfloat16>(const AArgs&);
template mla_status_t tc_attention<float>(const AArgs&, cudaStream_t, bool);
template mla_status_t tc_attention<double>(const AArgs&, cudaStream_t, bool);
template mla_status_t tc_attention<__half>(const AArgs&, cudaStream_t, bool);
template mla_status_t tc_attention<__nv_bfloat16>(const AArgs&, cudaStream_t, bool);

}  // namespace mla
