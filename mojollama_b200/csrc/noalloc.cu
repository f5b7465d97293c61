// mlq_matmul_q8act_noalloc: the Q8_0-activation matmul for callers that cannot allocate
// device memory.
//
// mlq_matmul_q8act expands the Q8_0 activations into fp32 in scratch memory taken from
// the library's arena (cudaMalloc on growth) and stages host buffers.  Some callers
// cannot let a library call cudaMalloc/cudaFree: a serving process that hands all of
// HBM to its own allocator at start-up (KV cache pools sized to the last byte), or a
// latency-critical decode loop that must not pay the device-wide synchronisation
// cudaFree implies.  This variant keeps its scratch in a fixed array in the library's
// own device image instead, and takes device pointers only, so it allocates nothing.
//
// Limits and sharing:
//   - at most kNoAllocMaxElems fp32 activation elements per call (B * n_cols);
//     larger calls are rejected with MLQ_ERR_CAPACITY before anything is launched.
//   - the scratch array exists once per device that loads the library and stays
//     resident until the process exits (256 KB + a 256-byte status word).
//   - every call on a device shares the array: calls that may overlap on the GPU
//     (different streams without ordering between them) race on it.  The array keeps
//     the last call's contents; each call overwrites every element it reads, so
//     nothing needs clearing.
//   - the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call before
//     any stream capture.
//   - the kernels' bounded waits report a wait that gave up in a status word of the same
//     static kind (not in the context status word mlq_device_status reads, which would
//     need an allocation to exist).  mlq_noalloc_status(stream) reads and clears it; it
//     allocates nothing either.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "mlq_internal.h"

namespace {

constexpr long long kNoAllocMaxElems = 65536;   // fp32 elements = 256 KB

// File-scope device scratch.  Host code must not use these names as addresses (in
// host code they are host-side stand-ins); it uses the addresses looked up below.
static __device__ __align__(256) float g_noalloc_act[kNoAllocMaxElems];
static __device__ __align__(256) int g_noalloc_status[64];

struct NoAllocDev {
    std::atomic<bool> ready{false};   // stored with release after the fields below are set
    float *act = nullptr;
    int *status = nullptr;
    int num_sms = 0;
};
constexpr int kMaxDev = 16;
NoAllocDev g_dev[kMaxDev];
std::mutex g_mu;

// Once per device, with that device current: device addresses of the scratch array
// and status word, and the SM count the launchers size their grids with.
bool setup_device(int dev, NoAllocDev &d) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (d.ready.load(std::memory_order_acquire)) return true;
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_act);
    if (e != cudaSuccess) {
        mlq::set_error(MLQ_ERR_CUDA, "mlq_matmul_q8act_noalloc: cudaGetSymbolAddress(scratch): %s",
                       cudaGetErrorString(e));
        return false;
    }
    void *q = nullptr;
    e = cudaGetSymbolAddress(&q, g_noalloc_status);
    if (e != cudaSuccess) {
        mlq::set_error(MLQ_ERR_CUDA, "mlq_matmul_q8act_noalloc: cudaGetSymbolAddress(status): %s",
                       cudaGetErrorString(e));
        return false;
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
        mlq::set_error(MLQ_ERR_CUDA, "mlq_matmul_q8act_noalloc: SM count: %s", cudaGetErrorString(e));
        return false;
    }
    d.act = static_cast<float *>(p);
    d.status = static_cast<int *>(q);
    d.num_sms = sms;
    d.ready.store(true, std::memory_order_release);
    return true;
}

// The current device's set-up record (set up on first use), or null with the error set.
NoAllocDev *current_device(const char *who) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
        cudaGetLastError();
        mlq::set_error(MLQ_ERR_NO_DEVICE, "%s: no current device", who);
        return nullptr;
    }
    NoAllocDev &d = g_dev[dev];
    if (!d.ready.load(std::memory_order_acquire) && !setup_device(dev, d)) return nullptr;
    return &d;
}

bool device_memory(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace

extern "C" int mlq_matmul_q8act_noalloc(const void *W, int qt, const uint8_t *x_q8, float *out, int n_rows,
                                        int n_cols, int B, void *stream) {
    using namespace mlq;
    if (!W || !x_q8 || !out || n_rows <= 0 || n_cols <= 0 || B <= 0 || n_cols % 32) {
        set_error(MLQ_ERR_ARG, "mlq_matmul_q8act_noalloc: null pointer, non-positive size or n_cols %% 32 != 0");
        return MLQ_ERR_ARG;
    }
    if ((long long)B * n_cols > kNoAllocMaxElems) {
        set_error(MLQ_ERR_CAPACITY,
                  "mlq_matmul_q8act_noalloc: B*n_cols = %lld exceeds the fixed scratch of %lld fp32 elements",
                  (long long)B * n_cols, kNoAllocMaxElems);
        return MLQ_ERR_CAPACITY;
    }
    // the same type check as mlq_matmul_q8act, before anything is launched
    if (mlq_row_bytes(qt, n_cols) == 0) {
        set_error(MLQ_ERR_TYPE, "mlq_matmul_q8act_noalloc: type %d with n_cols %d", qt, n_cols);
        return MLQ_ERR_TYPE;
    }
    if (!device_memory(W) || !device_memory(x_q8) || !device_memory(out)) {
        set_error(MLQ_ERR_ARG, "mlq_matmul_q8act_noalloc: W, x_q8 and out must be device memory");
        return MLQ_ERR_ARG;
    }
    NoAllocDev *dp = current_device("mlq_matmul_q8act_noalloc");
    if (!dp) return mlq_last_error();
    NoAllocDev &d = *dp;
    if (ref_compat() && qt == MLQ_MXFP4) qt = MLQ_MXFP4_REF;

    const LaunchEnv env{d.num_sms, d.status, true};
    LaunchEnvScope scope(&env);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const long long n = (long long)B * n_cols;
    int rc = launch_q8act_to_f32(x_q8, d.act, n, s);
    if (rc == MLQ_OK)
        rc = launch_matmul(static_cast<const uint8_t *>(W), qt, d.act, out, n_rows, n_cols, B,
                           mlq_row_bytes(qt, n_cols) * (size_t)n_rows, s);
    return rc;
}

// Status of the no-allocation calls on the current device: waits for `stream`, reads the
// status word their bounded waits write, clears it, and returns MLQ_ERR_TIMEOUT when a
// wait gave up (that call's output is then incomplete).  Allocates nothing.
extern "C" int mlq_noalloc_status(void *stream) {
    using namespace mlq;
    NoAllocDev *dp = current_device("mlq_noalloc_status");
    if (!dp) return mlq_last_error();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int h = 0;
    if (!MLQ_CUDA(cudaMemcpyAsync(&h, dp->status, sizeof(int), cudaMemcpyDeviceToHost, s))) return MLQ_ERR_CUDA;
    if (!MLQ_CUDA(cudaStreamSynchronize(s))) return MLQ_ERR_CUDA;
    if (h != 0) {
        if (!MLQ_CUDA(cudaMemsetAsync(dp->status, 0, sizeof(int), s))) return MLQ_ERR_CUDA;
        if (!MLQ_CUDA(cudaStreamSynchronize(s))) return MLQ_ERR_CUDA;
        set_error(MLQ_ERR_TIMEOUT, "mlq_noalloc_status: a device-side bounded wait gave up (code %d)", h);
        return MLQ_ERR_TIMEOUT;
    }
    return MLQ_OK;
}
