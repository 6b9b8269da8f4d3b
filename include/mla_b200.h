/*
 * mla_b200.h — C-ABI of the B200-native absorbed Multi-head Latent Attention
 * (MLA) decode layer-forward.
 *
 * The reference project (pgangwar-ucsd/mla-cuda) exposes this path as the
 * pybind11 module `mla_custom_cuda` with two functions:
 *
 *   q_absorbed(x, W_q_a, q_norm_w, W_q_b, W_uk, positions, nope_dim, rope_dim, eps)
 *       -> [q_absorbed, q_rope]            (mla_kernels.cu:599-608, bound at :1689-1690)
 *   mla_attention(q_absorbed, q_rope, c_kv, pe_cache, W_uv, scale) -> out
 *                                          (mla_kernels.cu:1479-1485, bound at :1691-1692)
 *
 * This header is the C boundary beneath the drop-in replacement of that module.
 * Every entry point takes raw device pointers to contiguous row-major arrays,
 * 64-bit sizes, a caller-owned workspace and a CUDA stream passed as `void*`
 * (a `cudaStream_t`; NULL is the legacy default stream). Nothing here
 * allocates device memory or synchronises the device: all work is enqueued on
 * the given stream, as the reference enqueues on the current torch stream
 * (mla_kernels.cu:667, :1549).
 *
 * Errors are returned as `mla_status_t`; `mla_last_error_message()` gives a
 * human-readable description of the most recent failure on the calling thread.
 * The Python shim turns any non-zero status into `RuntimeError`, which is what
 * the reference's TORCH_CHECK raises (mla_kernels.cu:627-635).
 */
#ifndef MLA_B200_H_
#define MLA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLA_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define MLA_API __attribute__((visibility("default")))
#else
#define MLA_API
#endif

typedef enum mla_status {
    MLA_OK = 0,
    MLA_ERR_INVALID_ARGUMENT = 1, /* bad shape, null pointer or inconsistent sizes   */
    MLA_ERR_UNSUPPORTED = 2,      /* dtype / precision / shape combination not built */
    MLA_ERR_WORKSPACE = 3,        /* workspace pointer null or smaller than required */
    MLA_ERR_CUDA = 4,             /* a CUDA runtime call or kernel launch failed     */
    MLA_ERR_DEVICE = 5            /* a kernel gave up on a bounded wait (see below)  */
} mla_status_t;

/* Storage dtype of every floating-point operand and output of one call. The
 * reference dispatches fp32/fp64/fp16 (AT_DISPATCH_FLOATING_TYPES_AND_HALF,
 * mla_kernels.cu:674, :1561); bf16 is new here. */
typedef enum mla_dtype {
    MLA_DTYPE_F32 = 0,
    MLA_DTYPE_F64 = 1,
    MLA_DTYPE_F16 = 2,
    MLA_DTYPE_BF16 = 3
} mla_dtype_t;

/* Arithmetic used by a call.
 *  MLA_PREC_EXACT : the accuracy of the accumulate dtype (fp64 for fp64
 *                   storage, fp32 otherwise), the reference's policy (AccType,
 *                   mla_kernels.cu:118-120). fp32 storage runs the contractions
 *                   on the tensor cores in 3xTF32 (fp32-class products, fp32
 *                   sums); fp16 / bf16 storage on the tensor cores in kind::f16
 *                   (16-bit products are exact in fp32, fp32 sums, the
 *                   probabilities carried as a 16-bit head plus remainder);
 *                   fp64 on CUDA cores. rel-L2 <= 1e-5 in fp32.
 *  MLA_PREC_TENSOR: tcgen05 tensor cores with bf16 operands and fp32
 *                   accumulation, scores never written to memory. fp32, fp16
 *                   and bf16 storage; rel-L2 <= 2e-2 against the fp32 path. */
typedef enum mla_precision {
    MLA_PREC_EXACT = 0,
    MLA_PREC_TENSOR = 1
} mla_precision_t;

/* ABI version of the loaded library (MLA_B200_ABI_VERSION at build time). */
MLA_API int mla_abi_version(void);

/* Static description of a status code. */
MLA_API const char* mla_status_string(mla_status_t status);

/* Message of the last failed call on this thread ("" if none). */
MLA_API const char* mla_last_error_message(void);

/* ---------------------------------------------------------------- Q-prep --
 * Replaces launch_q_absorbed (mla_kernels.cu:599-767): steps 2a1 (x @ W_q_a),
 * 2a-norm (RMSNorm with gain), 2a2 (@ W_q_b), 2b (RoPE, theta 10000,
 * interleaved pairs) and 2c (q_nope @ W_uk[h]).
 *
 *   x          [batch, sq, hidden]                 storage dtype
 *   W_q_a      [hidden, q_lora]
 *   q_norm_w   [q_lora]
 *   W_q_b      [q_lora, heads*(nope+rope)]
 *   W_uk       [heads, nope, kv_rank]
 *   positions  [sq] int64 on the device, absolute position of each query
 *   q_absorbed [batch, sq, heads, kv_rank]         output, storage dtype
 *   q_rope     [batch, sq, heads, rope]            output, storage dtype
 *
 * `rope` must be even. The workspace must hold at least the number of bytes
 * reported by mla_q_absorbed_workspace_size for the same arguments.
 */
MLA_API mla_status_t mla_q_absorbed_workspace_size(
    mla_dtype_t dtype, mla_precision_t precision,
    int64_t batch, int64_t sq, int64_t hidden, int64_t q_lora,
    int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank,
    size_t* bytes);

MLA_API mla_status_t mla_q_absorbed(
    mla_dtype_t dtype, mla_precision_t precision,
    const void* x, const void* W_q_a, const void* q_norm_w,
    const void* W_q_b, const void* W_uk, const int64_t* positions,
    int64_t batch, int64_t sq, int64_t hidden, int64_t q_lora,
    int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank,
    double eps,
    void* q_absorbed, void* q_rope,
    void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------- pre-packed Q weights --
 * Beside the drop-in (the reference converts nothing; its callers pass the
 * fp32 weights, made contiguous, on every call: exhaustive_benchmark_suite.py:
 * 261-265, stage_profile.py:57-63). For fp32 storage in tensor precision, the
 * Q-prep weights W_q_a, W_q_b and W_uk can be converted once, at weight-load
 * time, to one bf16 buffer of mla_pack_q_weights_size() bytes; then
 * mla_q_absorbed_packed computes q_absorbed / q_rope from it, streaming half the
 * weight bytes of mla_q_absorbed with MLA_PREC_TENSOR (bf16 operands, fp32
 * accumulation, fp32 RMSNorm and RoPE; rel-L2 <= 2e-2). x, q_norm_w, positions
 * and the outputs are as for mla_q_absorbed (fp32). The packed buffer stays
 * valid as long as the weights do not change.
 */
MLA_API mla_status_t mla_pack_q_weights_size(
    mla_dtype_t dtype, int64_t hidden, int64_t q_lora, int64_t heads,
    int64_t nope, int64_t rope, int64_t kv_rank, size_t* bytes);

MLA_API mla_status_t mla_pack_q_weights(
    mla_dtype_t dtype, const void* W_q_a, const void* W_q_b, const void* W_uk,
    int64_t hidden, int64_t q_lora, int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank,
    void* packed, size_t packed_bytes, void* stream);

MLA_API mla_status_t mla_q_absorbed_packed_workspace_size(
    mla_dtype_t dtype, int64_t batch, int64_t sq, int64_t hidden, int64_t q_lora,
    int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank, size_t* bytes);

MLA_API mla_status_t mla_q_absorbed_packed(
    mla_dtype_t dtype, const void* x, const void* packed, const void* q_norm_w,
    const int64_t* positions, int64_t batch, int64_t sq, int64_t hidden, int64_t q_lora,
    int64_t heads, int64_t nope, int64_t rope, int64_t kv_rank, double eps,
    void* q_absorbed, void* q_rope, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- attention --
 * Replaces launch_mla_attention (mla_kernels.cu:1479-1682): scores
 * (q_absorbed . c_kv + q_rope . pe_cache) / scale, softmax over the keys,
 * ctx = P @ c_kv, out = ctx @ W_uv[h]^T.
 *
 *   q_absorbed [batch, sq, heads, kv_rank]
 *   q_rope     [batch, sq, heads, rope]
 *   c_kv       [batch, sk, kv_rank]
 *   pe_cache   [batch, sk, rope]           shared by all heads
 *   W_uv       [heads, v_dim, kv_rank]
 *   out        [batch, sq, heads, v_dim]   output, storage dtype
 *
 * `scale` divides the scores (the reference passes sqrt(192), not its
 * reciprocal: mla_kernels.cu:851). `causal` = 0 is the reference's semantics
 * (every query attends all sk keys); 1 lets query i of sq attend keys
 * 0 .. sk-sq+i only (requires sk >= sq). sk == 0 yields zeros.
 */
MLA_API mla_status_t mla_attention_workspace_size(
    mla_dtype_t dtype, mla_precision_t precision,
    int64_t batch, int64_t sq, int64_t sk, int64_t heads,
    int64_t kv_rank, int64_t rope, int64_t v_dim, int causal,
    size_t* bytes);

MLA_API mla_status_t mla_attention(
    mla_dtype_t dtype, mla_precision_t precision,
    const void* q_absorbed, const void* q_rope,
    const void* c_kv, const void* pe_cache, const void* W_uv,
    int64_t batch, int64_t sq, int64_t sk, int64_t heads,
    int64_t kv_rank, int64_t rope, int64_t v_dim,
    double scale, int causal,
    void* out,
    void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------- pre-packed W_uv ---------
 * Beside the drop-in, like mla_pack_q_weights. For fp32 storage in tensor
 * precision, W_uv [heads, v_dim, kv_rank] can be converted once to bf16 (a
 * buffer of mla_pack_uv_weights_size() bytes, same layout); then
 * mla_attention_packed_uv runs mla_attention with MLA_PREC_TENSOR, keeping the
 * normalised context in bf16 and projecting it with the bf16 W_uv (kind::f16,
 * fp32 accumulation, fp32 output): the 3d step streams half the bytes.
 * Operands, workspace (mla_attention_workspace_size with MLA_PREC_TENSOR) and
 * output are those of mla_attention; dtype must be MLA_DTYPE_F32 and the shape
 * one the tensor-core attention covers (heads 128, kv_rank 512, rope 64, v_dim
 * a multiple of 32), else MLA_ERR_UNSUPPORTED.
 */
MLA_API mla_status_t mla_pack_uv_weights_size(
    mla_dtype_t dtype, int64_t heads, int64_t v_dim, int64_t kv_rank, size_t* bytes);

MLA_API mla_status_t mla_pack_uv_weights(
    mla_dtype_t dtype, const void* W_uv, int64_t heads, int64_t v_dim, int64_t kv_rank,
    void* packed, size_t packed_bytes, void* stream);

MLA_API mla_status_t mla_attention_packed_uv(
    mla_dtype_t dtype,
    const void* q_absorbed, const void* q_rope,
    const void* c_kv, const void* pe_cache, const void* W_uv_packed,
    int64_t batch, int64_t sq, int64_t sk, int64_t heads,
    int64_t kv_rank, int64_t rope, int64_t v_dim,
    double scale, int causal,
    void* out,
    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- KV-cache write --
 * The step upstream of the decode read. The reference has no kernel for it
 * (its caches are inputs; the write is only mentioned,
 * exhaustive_benchmark_suite.py:189); the arithmetic composes the reference's
 * own rmsnorm (:252-258) and apply_rope (:210-232). For each new token (b, s):
 *
 *   kv = x[b, s] @ W_kv_a                               [kv_rank + rope]
 *   c_kv    [b, slots[s]] = RMSNorm(kv[:kv_rank]) * kv_norm_w   (eps)
 *   pe_cache[b, slots[s]] = RoPE(kv[kv_rank:], positions[s])    (theta 10000,
 *                                                                interleaved pairs)
 *
 *   x          [batch, sq, hidden]        storage dtype (fp32, fp16 or bf16)
 *   W_kv_a     [hidden, kv_rank + rope]
 *   kv_norm_w  [kv_rank]
 *   positions, slots  [sq] int64 on the device (same for every sequence)
 *   c_kv       [batch, capacity, kv_rank]  written in place at the slots
 *   pe_cache   [batch, capacity, rope]
 *
 * Exact precision projects in 3xTF32 (fp32 storage); tensor precision in
 * kind::tf32; 16-bit storage in kind::f16 (fp32 accumulation either way). A
 * slot outside [0, capacity) is not written and records code 950 in the device
 * status (mla_device_status).
 */
MLA_API mla_status_t mla_kv_cache_write_workspace_size(
    mla_dtype_t dtype, mla_precision_t precision, int64_t batch, int64_t sq,
    int64_t hidden, int64_t kv_rank, int64_t rope, size_t* bytes);

MLA_API mla_status_t mla_kv_cache_write(
    mla_dtype_t dtype, mla_precision_t precision,
    const void* x, const void* W_kv_a, const void* kv_norm_w,
    const int64_t* positions, const int64_t* slots,
    int64_t batch, int64_t sq, int64_t hidden, int64_t kv_rank, int64_t rope,
    int64_t capacity, double eps,
    void* c_kv, void* pe_cache, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------ key-sharded attention --
 * No counterpart in the reference (it is single-GPU). For long contexts the
 * keys of every sequence can be split across GPUs: each GPU runs
 * mla_attention_partial on its key shard, the shards' outputs and lse are
 * gathered (NCCL all-gather), and mla_lse_combine merges them. The merge is
 * exact because the W_uv projection is linear in the normalised context.
 *
 * mla_attention_partial: same operands, workspace and semantics as
 * mla_attention (without causal masking), plus
 *   lse  [batch, sq, heads] fp32: natural-log sum of exp(score / scale) over
 *        this shard's keys (-inf for an empty shard).
 * mla_lse_combine: outs [parts, rows, v_dim] and lses [parts, rows] (rows =
 * batch*sq*heads) -> out [rows, v_dim] (and lse_out [rows] if not NULL);
 * fp32 / fp16 / bf16.
 */
MLA_API mla_status_t mla_attention_partial(
    mla_dtype_t dtype, mla_precision_t precision,
    const void* q_absorbed, const void* q_rope,
    const void* c_kv, const void* pe_cache, const void* W_uv,
    int64_t batch, int64_t sq, int64_t sk, int64_t heads,
    int64_t kv_rank, int64_t rope, int64_t v_dim,
    double scale,
    void* out, float* lse,
    void* workspace, size_t workspace_bytes, void* stream);

MLA_API mla_status_t mla_lse_combine(
    mla_dtype_t dtype, int64_t parts, int64_t rows, int64_t v_dim,
    const void* outs, const float* lses,
    void* out, float* lse_out, void* stream);

/* ------------------------------------------------- allocation-free variant --
 * No counterpart in the reference. Same computation as mla_attention with
 * MLA_PREC_TENSOR (fp32, fp16 or bf16 storage; heads 128, kv_rank 512,
 * rope 64), for callers that cannot allocate device memory when they call:
 * a server whose memory pool already owns the GPU, or code running where
 * cudaMalloc may not be called. The workspace is a fixed device array of
 * mla_attention_noalloc_max_scratch() bytes (96 MiB) that exists on every
 * GPU where the library is loaded, until the process exits; shapes that need
 * more return MLA_ERR_WORKSPACE. Nothing is allocated or freed.
 *
 * The first call on a device looks up that array's device address (once per
 * device, with the device current); make that first call before any stream
 * capture. All calls share the one array and it keeps the last call's
 * contents, so calls that overlap on the GPU (different streams or threads)
 * race: serialise them.
 */
MLA_API mla_status_t mla_attention_noalloc(
    mla_dtype_t dtype,
    const void* q_absorbed, const void* q_rope,
    const void* c_kv, const void* pe_cache, const void* W_uv,
    int64_t batch, int64_t sq, int64_t sk, int64_t heads,
    int64_t kv_rank, int64_t rope, int64_t v_dim,
    double scale, int causal,
    void* out, void* stream);

/* ------------------------------------------------------ device failure status --
 * No counterpart in the reference, whose kernels can only hang or succeed
 * (its host reports launch and shared-memory opt-in failures,
 * mla_kernels.cu:141-146). Every mbarrier wait of this library's tensor-core
 * kernels is bounded by wall time (2 s by default). A wait that runs out
 * records a non-zero code in a per-device status block (the first code
 * wins), and the kernel drains its in-flight copies and MMAs, frees its TMEM
 * and returns; the outputs of that call are invalid. The code stays set until
 * cleared.
 *
 * mla_device_status: waits for `stream`, reads the code of the current
 *   device into *code, and returns MLA_ERR_DEVICE if it is non-zero.
 * mla_device_status_clear: enqueues a reset of the code on `stream`.
 * mla_set_wait_limit_ns: sets the wait bound of later launches on the
 *   current device (0 restores the default); synchronises `stream`.
 * mla_wait_selftest: launches a kernel whose one bounded wait is on a barrier
 *   that nothing completes, so it runs out after the wait limit and records
 *   code 900. Used by tests to check the reporting path.
 */
MLA_API mla_status_t mla_device_status(void* stream, int* code);
MLA_API mla_status_t mla_device_status_clear(void* stream);
MLA_API mla_status_t mla_set_wait_limit_ns(uint64_t ns, void* stream);
MLA_API mla_status_t mla_wait_selftest(void* stream);

/* ------------------------------------------------------------ kernel timing --
 * Benchmark hook (no counterpart in the reference, which times stages with
 * CUDA events from Python, stage_profile.py:31-41). While enabled, every launch
 * of the tensor-core decode-attention kernel is bracketed by a CUDA event pair
 * on its stream (at most 8192 launches are kept). mla_timing_read waits for
 * the recorded launches, returns their summed device time and count, and
 * starts a new count. Do not enable it during CUDA graph capture.
 */
MLA_API mla_status_t mla_timing_enable(int on);
MLA_API mla_status_t mla_timing_read(double* total_ms, int64_t* launches);

/* Size in bytes of the fixed scratch array used by mla_attention_noalloc. */
MLA_API size_t mla_attention_noalloc_max_scratch(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MLA_B200_H_ */
