// Device-side failure status of the library's kernels.
//
// Every tensor-core kernel bounds its mbarrier waits by wall time. A wait that
// runs out records a code in one status block per device (first code wins),
// raises the kernel's shared abort flag, and the kernel drains and returns; it
// never traps. The host reads the block with mla_device_status(), after the
// work it wants to check has finished on the stream; the code stays set until
// mla_device_status_clear(). The same block carries the wait limit, so a test
// can shorten it (mla_set_wait_limit_ns) and make a wait run out on purpose.
//
// The reference reports only host-side failures (TORCH_CHECK and the
// shared-memory opt-in check, mla_kernels.cu:141-146); a kernel that stalls
// there hangs the device.
#include "common.cuh"
#include "sm100.cuh"

#include <mutex>

namespace mla {

namespace {

__device__ __align__(16) DeviceStatus g_device_status = {0, 0, sm100::kWaitLimitNs};

constexpr int kMaxDevices = 64;
DeviceStatus* g_status_ptr[kMaxDevices] = {nullptr};
std::mutex g_status_mu;

// A kernel whose only job is to wait, with the library's bounded wait, on an
// mbarrier that nothing arrives on. It exercises the timeout path (code,
// abort flag, return) without any other work in flight.
__global__ void wait_selftest_kernel(DeviceStatus* status) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bar, 1);
        abort_flag = 0;
        sm100::fence_mbar_init();
    }
    __syncthreads();
    // parity 0 completes only when the one expected arrival happens; none does
    sm100::mbar_wait(&bar, 0, &abort_flag, &status->code, kErrSelftestTimeout);
}

}  // namespace

mla_status_t device_status_block(DeviceStatus** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return set_error(MLA_ERR_CUDA, "MLA: no usable current device");
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (!g_status_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_device_status);
        if (e != cudaSuccess || !p)
            return set_error(MLA_ERR_CUDA, "MLA: cudaGetSymbolAddress of the status block failed: %s",
                             cudaGetErrorString(e));
        g_status_ptr[dev] = static_cast<DeviceStatus*>(p);
    }
    *out = g_status_ptr[dev];
    return MLA_OK;
}

// ------------------------------------------------------------------ timing
// Optional CUDA-event timing of the decode-attention kernel alone (the kernel
// that bounds the layer), for benchmarks that report its roofline fraction.
// Off by default; when on, each launch records an event pair on its stream.
namespace {
constexpr int kMaxTimed = 8192;
struct Timing {
    bool on = false;
    int n = 0;
    cudaEvent_t ev[2 * kMaxTimed] = {};
    int created = 0;
} g_timing;
std::mutex g_timing_mu;
}  // namespace

void timing_mark(cudaStream_t st, bool begin) {
    std::lock_guard<std::mutex> lock(g_timing_mu);
    if (!g_timing.on || g_timing.n >= kMaxTimed) return;
    const int k = 2 * g_timing.n + (begin ? 0 : 1);
    if (k >= g_timing.created) {
        if (cudaEventCreate(&g_timing.ev[k]) != cudaSuccess) return;
        g_timing.created = k + 1;
    }
    cudaEventRecord(g_timing.ev[k], st);
    if (!begin) ++g_timing.n;
}

}  // namespace mla

using namespace mla;

extern "C" {

mla_status_t mla_device_status(void* stream, int* code) {
    if (!code) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: code must not be NULL");
    DeviceStatus* s = nullptr;
    MLA_TRY(device_status_block(&s));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int v = 0;
    if (cudaMemcpyAsync(&v, &s->code, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return set_error(MLA_ERR_CUDA, "MLA: reading the device status failed: %s",
                         cudaGetErrorString(cudaGetLastError()));
    *code = v;
    if (v != 0)
        return set_error(MLA_ERR_DEVICE,
                         "MLA: device-side failure (code %d: %s); the outputs of that call are invalid", v,
                         v == 950 ? "KV-cache write: slot outside the cache, not written"
                         : v >= kErrSelftestTimeout ? "wait self-test" : v >= 200 ? "tensor-core GEMM"
                                                                                   : "decode attention");
    return MLA_OK;
}

mla_status_t mla_device_status_clear(void* stream) {
    DeviceStatus* s = nullptr;
    MLA_TRY(device_status_block(&s));
    if (cudaMemsetAsync(&s->code, 0, sizeof(int), static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return set_error(MLA_ERR_CUDA, "MLA: clearing the device status failed");
    return MLA_OK;
}

mla_status_t mla_set_wait_limit_ns(uint64_t ns, void* stream) {
    DeviceStatus* s = nullptr;
    MLA_TRY(device_status_block(&s));
    const uint64_t v = ns == 0 ? sm100::kWaitLimitNs : ns;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&s->wait_limit_ns, &v, sizeof(v), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return set_error(MLA_ERR_CUDA, "MLA: setting the wait limit failed");
    return MLA_OK;
}

mla_status_t mla_wait_selftest(void* stream) {
    DeviceStatus* s = nullptr;
    MLA_TRY(device_status_block(&s));
    wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(s);
    return check_launch("wait self-test");
}

mla_status_t mla_timing_enable(int on) {
    std::lock_guard<std::mutex> lock(g_timing_mu);
    g_timing.on = on != 0;
    g_timing.n = 0;
    return MLA_OK;
}

mla_status_t mla_timing_read(double* total_ms, int64_t* launches) {
    if (!total_ms || !launches) return set_error(MLA_ERR_INVALID_ARGUMENT, "MLA: null output pointer");
    std::lock_guard<std::mutex> lock(g_timing_mu);
    double tot = 0.0;
    for (int i = 0; i < g_timing.n; ++i) {
        float ms = 0.f;
        if (cudaEventSynchronize(g_timing.ev[2 * i + 1]) != cudaSuccess ||
            cudaEventElapsedTime(&ms, g_timing.ev[2 * i], g_timing.ev[2 * i + 1]) != cudaSuccess)
            return set_error(MLA_ERR_CUDA, "MLA: reading the kernel timing events failed");
        tot += ms;
    }
    *total_ms = tot;
    *launches = g_timing.n;
    g_timing.n = 0;
    return MLA_OK;
}

}  // extern "C"
