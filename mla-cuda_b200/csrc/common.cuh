// Shared definitions for the MLA B200 kernels: dtype traits, status plumbing,
// small math helpers. Everything here is header-only and device/host neutral.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include <utility>

#include "mla_b200.h"

namespace mla {

// Accumulate dtype policy: fp64 storage accumulates in fp64, every other
// storage dtype in fp32. Same policy as the reference's AccType
// (mla_kernels.cu:118-120), extended to bf16.
template <typename T> struct AccOf { using type = float; };
template <> struct AccOf<double> { using type = double; };
template <typename T> using acc_t = typename AccOf<T>::type;

template <typename To, typename From>
__device__ __forceinline__ To cvt(From v) { return static_cast<To>(v); }
template <> __device__ __forceinline__ float cvt<float, __half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float cvt<float, __nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ __half cvt<__half, float>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16, float>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float fexp(float x) { return expf(x); }
__device__ __forceinline__ double fexp(double x) { return exp(x); }

template <typename A> __device__ __forceinline__ A neg_inf();
template <> __device__ __forceinline__ float neg_inf<float>() { return -__int_as_float(0x7f800000); }
template <> __device__ __forceinline__ double neg_inf<double>() { return -__longlong_as_double(0x7ff0000000000000LL); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Per-device failure status of the kernels (status.cu). `code` is the first
// bounded-wait timeout code recorded (0 = none); `wait_limit_ns` bounds every
// mbarrier wait. Kernels get a pointer to `code`; the limit sits 8 bytes after it.
struct DeviceStatus {
    int code;
    int reserved;
    unsigned long long wait_limit_ns;
};
constexpr int kErrSelftestTimeout = 900;

// Device address of this device's status block (looked up once per device).
mla_status_t device_status_block(DeviceStatus** out);

// Benchmark hook: an event pair around the decode-attention kernel when
// mla_timing_enable(1) is in effect (status.cu).
void timing_mark(cudaStream_t st, bool begin);

// Records a message for mla_last_error_message() and returns the status.
mla_status_t set_error(mla_status_t st, const char* fmt, ...);

// Checks the launch that just happened on this thread.
mla_status_t check_launch(const char* what);

// Number of SMs of the current device, cached per device.
int sm_count();

// Programmatic dependent launch. The layer's kernels are launched with the
// programmatic-serialization attribute, so a kernel's CTAs may start while its
// predecessor on the stream is still finishing. Each such kernel does only
// setup that touches no global data (barriers, TMEM, tensor-map prefetch,
// L2 prefetch hints) before pdl_wait(), which returns once the predecessor has
// completed and its writes are visible; it then lets its own dependents launch
// (pdl_trigger). Every kernel launched this way waits before it completes, so
// all earlier work on the stream is complete once a kernel has passed its wait.
// Outside such a launch both are no-ops. MLA_PDL=0 launches without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace mla

#define MLA_TRY(expr)                                  \
    do {                                               \
        mla_status_t _st = (expr);                     \
        if (_st != MLA_OK) return _st;                 \
    } while (0)
