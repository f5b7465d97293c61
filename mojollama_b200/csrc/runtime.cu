// Runtime of libmojollama_b200.so: device contexts, the library stream, the
// thread-local error state, host-pointer staging and the weight residency cache.
//
// The reference C engine is called with host pointers from numpy
// (src/mojollama/kernels/turbo_engine_v7_moe.py:240-423 of the reference) and
// returns when its outputs are written.  Here a host weight buffer is copied to
// HBM once and kept (keyed by address and size, like the reference's weights
// that stay mmapped for the life of the engine), activations are staged through
// a per-device arena, and a call that touched host memory synchronises before
// returning.  Calls whose pointers are all device memory stay asynchronous.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <vector>

#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

// ------------------------------------------------------------------------------ errors
static thread_local int t_err = MLQ_OK;
static thread_local char t_msg[512] = {0};

void set_error(int code, const char *fmt, ...) {
    t_err = code;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    if (getenv("MLQ_VERBOSE")) fprintf(stderr, "[mojollama_b200] error %d: %s\n", code, t_msg);
}

// ------------------------------------------------------------------------------ contexts
static const int kMaxDev = 16;
static Ctx g_ctx[kMaxDev];
static std::mutex g_mu;
static thread_local int t_dev = -1;
static std::atomic<unsigned long long> g_launches{0};
static std::atomic<int> g_compat{-1};

void count_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

bool ref_compat() {
    int v = g_compat.load();
    if (v < 0) {
        const char *e = getenv("MLQ_REF_COMPAT");
        v = (e && atoi(e) != 0) ? 1 : 0;
        g_compat.store(v);
    }
    return v != 0;
}

static bool init_device(int dev) {
    if (dev < 0 || dev >= kMaxDev) {
        set_error(MLQ_ERR_ARG, "device %d out of range", dev);
        return false;
    }
    Ctx &c = g_ctx[dev];
    if (c.device == dev) return true;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= dev) {
        cudaGetLastError();
        set_error(MLQ_ERR_NO_DEVICE, "no CUDA device %d (count %d)", dev, n);
        return false;
    }
    if (!MLQ_CUDA(cudaSetDevice(dev))) return false;
    int sms = 0;
    if (!MLQ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))) return false;
    cudaStream_t s = nullptr;
    if (!MLQ_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking))) return false;
    // the status word lives in mapped pinned host memory: kernels write it over PCIe (only
    // when a bounded wait gives up) and the host reads it after any synchronisation
    int *hst = nullptr, *st = nullptr;
    if (!MLQ_CUDA(cudaHostAlloc((void **)&hst, 64, cudaHostAllocMapped | cudaHostAllocPortable))) return false;
    memset(hst, 0, 64);
    if (!MLQ_CUDA(cudaHostGetDevicePointer((void **)&st, hst, 0))) return false;
    c.num_sms = sms;
    c.own_stream = s;
    c.stream = s;
    c.d_status = st;
    c.h_status = hst;
    c.device = dev;
    return true;
}

// After a synchronisation: MLQ_ERR_TIMEOUT (and the word cleared) when a device-side
// bounded wait gave up since the last check, else MLQ_OK.
static int take_device_status(Ctx *c) {
    const int h = c->h_status[0];
    if (h == 0) return MLQ_OK;
    c->h_status[0] = 0;
    set_error(MLQ_ERR_TIMEOUT, "device-side bounded wait gave up (code 0x%x)", h);
    return MLQ_ERR_TIMEOUT;
}

Ctx *ctx() {
    if (t_dev < 0) {
        int d = 0;
        if (cudaGetDevice(&d) != cudaSuccess) { cudaGetLastError(); d = 0; }
        t_dev = d;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!init_device(t_dev)) return nullptr;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != t_dev) cudaSetDevice(t_dev);
    return &g_ctx[t_dev];
}

cudaStream_t stream() {
    Ctx *c = ctx();
    return c ? c->stream : nullptr;
}

static thread_local const LaunchEnv *t_env_override = nullptr;
static thread_local LaunchEnv t_env_ctx;

const LaunchEnv *launch_env() {
    if (t_env_override) return t_env_override;
    Ctx *c = ctx();
    if (!c) return nullptr;
    t_env_ctx.num_sms = c->num_sms;
    t_env_ctx.d_status = c->d_status;
    return &t_env_ctx;
}

LaunchEnvScope::LaunchEnvScope(const LaunchEnv *e) : prev(t_env_override) { t_env_override = e; }
LaunchEnvScope::~LaunchEnvScope() { t_env_override = prev; }

int *dev_status() {
    Ctx *c = ctx();
    return c ? c->d_status : nullptr;
}

bool is_device_ptr(const void *p) {
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// ------------------------------------------------------------------------------ residency cache
// Each entry keeps a content sample of the host buffer (all of it up to 16 KB; else
// the first and last 4 KB and 64 evenly spaced 64-byte windows).  A hit whose sample
// no longer matches -- a freed host buffer re-allocated at the same address with the
// same size, or weights rewritten in place -- re-uploads the buffer.  Changes that
// touch none of the sampled bytes are not seen: treat host weights as immutable
// after first use, or call mlq_cache_clear().
struct CacheEntry { void *dev; size_t bytes; std::vector<uint8_t> sample; };
static std::map<std::pair<uintptr_t, size_t>, CacheEntry> g_cache[kMaxDev];
static size_t g_cache_bytes[kMaxDev];

static void take_sample(const uint8_t *h, size_t bytes, std::vector<uint8_t> &s) {
    if (bytes <= 16384) {
        s.assign(h, h + bytes);
        return;
    }
    s.resize(8192 + 64 * 64);
    memcpy(s.data(), h, 4096);
    memcpy(s.data() + 4096, h + bytes - 4096, 4096);
    const size_t stride = (bytes - 64) / 64;
    for (int i = 0; i < 64; i++) memcpy(s.data() + 8192 + 64 * i, h + stride * i, 64);
}

static bool sample_matches(const uint8_t *h, size_t bytes, const std::vector<uint8_t> &s) {
    if (bytes <= 16384) return memcmp(h, s.data(), bytes) == 0;
    if (memcmp(h, s.data(), 4096) || memcmp(h + bytes - 4096, s.data() + 4096, 4096)) return false;
    const size_t stride = (bytes - 64) / 64;
    for (int i = 0; i < 64; i++)
        if (memcmp(h + stride * i, s.data() + 8192 + 64 * i, 64)) return false;
    return true;
}

// Whole host tensors registered with mlq_register_weights: any pointer inside one
// (e.g. one expert of a 3-D expert tensor) maps to the same offset of its device copy.
// Each range keeps a small content sample (first/last 64 bytes and 16 spread 16-byte
// windows, 384 bytes) checked on every lookup, so a range whose host memory was freed
// and reused for other data is re-uploaded instead of serving a stale copy.
struct RangeEntry { size_t bytes; void *dev; std::vector<uint8_t> sample; };
static std::map<uintptr_t, RangeEntry> g_ranges[kMaxDev];

static void range_sample(const uint8_t *h, size_t bytes, std::vector<uint8_t> &s) {
    if (bytes <= 384) {
        s.assign(h, h + bytes);
        return;
    }
    s.resize(384);
    memcpy(s.data(), h, 64);
    memcpy(s.data() + 64, h + bytes - 64, 64);
    const size_t stride = (bytes - 16) / 16;
    for (int i = 0; i < 16; i++) memcpy(s.data() + 128 + 16 * i, h + stride * i, 16);
}

static const void *in_registered_range(int dev, const void *host, size_t bytes) {
    auto &m = g_ranges[dev];
    const uintptr_t p = (uintptr_t)host;
    auto it = m.upper_bound(p);
    if (it == m.begin()) return nullptr;
    --it;
    if (p + bytes > it->first + it->second.bytes) return nullptr;
    std::vector<uint8_t> now;
    range_sample((const uint8_t *)it->first, it->second.bytes, now);
    if (now != it->second.sample) {
        if (cudaMemcpy(it->second.dev, (const void *)it->first, it->second.bytes, cudaMemcpyHostToDevice) !=
            cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        it->second.sample.swap(now);
    }
    return (const char *)it->second.dev + (p - it->first);
}

static const void *resident(const void *host, size_t bytes) {
    Ctx *c = ctx();
    if (!c) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (const void *r = in_registered_range(c->device, host, bytes)) return r;
    auto key = std::make_pair((uintptr_t)host, bytes);
    auto &m = g_cache[c->device];
    auto it = m.find(key);
    const uint8_t *h = (const uint8_t *)host;
    if (it != m.end()) {
        if (sample_matches(h, bytes, it->second.sample)) return it->second.dev;
        if (!MLQ_CUDA(cudaMemcpyAsync(it->second.dev, host, bytes, cudaMemcpyHostToDevice, c->stream)))
            return nullptr;
        take_sample(h, bytes, it->second.sample);
        return it->second.dev;
    }
    void *d = nullptr;
    // pad so that 16-byte vector reads of the last block stay inside the allocation
    if (!MLQ_CUDA(cudaMalloc(&d, bytes + 256))) return nullptr;
    if (!MLQ_CUDA(cudaMemcpyAsync(d, host, bytes, cudaMemcpyHostToDevice, c->stream))) {
        cudaFree(d);
        return nullptr;
    }
    cudaMemsetAsync((char *)d + bytes, 0, 256, c->stream);
    CacheEntry e{d, bytes, {}};
    take_sample(h, bytes, e.sample);
    m[key] = std::move(e);
    g_cache_bytes[c->device] += bytes;
    return d;
}

// ------------------------------------------------------------------------------ staging arena
struct Arena {
    std::vector<std::pair<char *, size_t>> chunks;   // [0] is the main chunk
    size_t off = 0;                                  // offset in the last chunk
    int depth = 0;
};
static Arena g_arena[kMaxDev];

static void arena_begin(Ctx *c) {
    Arena &a = g_arena[c->device];
    if (a.depth++ > 0) return;
    if (a.chunks.size() > 1) {
        // grew during the previous call: wait for its work, then consolidate
        cudaStreamSynchronize(c->stream);
        size_t total = 0;
        for (auto &ch : a.chunks) { total += ch.second; cudaFree(ch.first); }
        a.chunks.clear();
        char *p = nullptr;
        if (cudaMalloc(&p, total) == cudaSuccess) a.chunks.push_back({p, total});
        else cudaGetLastError();
    }
    a.off = 0;
}

static void arena_end(Ctx *c) {
    Arena &a = g_arena[c->device];
    if (a.depth > 0) a.depth--;
}

static void *arena_alloc(Ctx *c, size_t bytes) {
    Arena &a = g_arena[c->device];
    bytes = (bytes + 255) & ~(size_t)255;
    if (!a.chunks.empty() && a.off + bytes <= a.chunks.back().second) {
        void *p = a.chunks.back().first + a.off;
        a.off += bytes;
        return p;
    }
    size_t want = bytes < ((size_t)64 << 20) ? ((size_t)64 << 20) : bytes;
    char *p = nullptr;
    if (!MLQ_CUDA(cudaMalloc(&p, want))) return nullptr;
    a.chunks.push_back({p, want});
    a.off = bytes;
    return p;
}

CallScope::CallScope() {
    Ctx *c = ctx();
    if (!c) { failed = true; return; }
    arena_begin(c);
}

CallScope::~CallScope() {
    Ctx *c = ctx();
    if (c) arena_end(c);
}

void *CallScope::stage(size_t bytes) {
    Ctx *c = ctx();
    if (!c) { failed = true; return nullptr; }
    void *p = arena_alloc(c, bytes ? bytes : 1);
    if (!p) failed = true;
    return p;
}

// Small inputs in pinned host memory: one kernel reads them over PCIe into the staging
// buffer.  It lets the next kernel launch at once (programmatic dependent launch), so a
// GEMV starts streaming its weights while the input is still crossing; the GEMV reads the
// input only after its dependency wait.  A copy-engine transfer can overlap nothing.
static constexpr size_t kPinnedKernelCopyMax = 256 * 1024;

__global__ void __launch_bounds__(256) k_copy_pinned(uint8_t *__restrict__ dst, const uint8_t *__restrict__ src,
                                                     size_t n) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x, step = (size_t)gridDim.x * blockDim.x;
    if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0) {
        for (size_t i = i0; 16 * i < n; i += step) {
            if (16 * i + 16 <= n) {
                reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(src)[i];
            } else {
                for (size_t b = 16 * i; b < n; b++) dst[b] = src[b];
            }
        }
    } else {
        for (size_t b = i0; b < n; b += step) dst[b] = src[b];
    }
}

const void *CallScope::in(const void *p, size_t bytes) {
    if (failed || !p) return nullptr;
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, p) != cudaSuccess) {
        cudaGetLastError();
        pa.type = cudaMemoryTypeUnregistered;
    }
    if (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged) return p;
    any_host = true;
    void *d = stage(bytes);
    if (!d) return nullptr;
    void *hp = nullptr;
    if (bytes && bytes <= kPinnedKernelCopyMax && pa.type == cudaMemoryTypeHost &&
        cudaHostGetDevicePointer(&hp, const_cast<void *>(p), 0) == cudaSuccess && hp) {
        const unsigned grid = (unsigned)((bytes + 4095) / 4096);
        k_copy_pinned<<<grid, 256, 0, stream()>>>((uint8_t *)d, (const uint8_t *)hp, bytes);
        count_launch();
        if (!MLQ_CUDA(cudaGetLastError())) {
            failed = true;
            return nullptr;
        }
        return d;
    }
    cudaGetLastError();
    if (bytes && !MLQ_CUDA(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, stream()))) {
        failed = true;
        return nullptr;
    }
    return d;
}

void *CallScope::out(void *p, size_t bytes) {
    if (failed || !p) return nullptr;
    if (is_device_ptr(p)) return p;
    any_host = true;
    void *d = stage(bytes);
    if (!d) return nullptr;
    if (n_pending_ >= 64) { set_error(MLQ_ERR_CAPACITY, "too many host outputs"); failed = true; return nullptr; }
    pending_[n_pending_++] = Pending{p, d, bytes};
    return d;
}

void *CallScope::out_direct(void *p, size_t bytes, bool *host_mapped) {
    *host_mapped = false;
    if (failed || !p) return nullptr;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return out(p, bytes);
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return p;
    void *d = nullptr;
    if (a.type == cudaMemoryTypeHost && cudaHostGetDevicePointer(&d, p, 0) == cudaSuccess && d) {
        any_host = true;   // finish() synchronises before the caller reads it
        *host_mapped = true;
        return d;
    }
    cudaGetLastError();
    return out(p, bytes);
}

void *CallScope::inout(void *p, size_t bytes) {
    if (failed || !p) return nullptr;
    if (is_device_ptr(p)) return p;
    void *d = const_cast<void *>(in(p, bytes));
    if (!d) return nullptr;
    if (n_pending_ >= 64) { set_error(MLQ_ERR_CAPACITY, "too many host outputs"); failed = true; return nullptr; }
    pending_[n_pending_++] = Pending{p, d, bytes};
    return d;
}

void *CallScope::scratch(size_t bytes) { return failed ? nullptr : stage(bytes); }

const void *CallScope::weights(const void *p, size_t bytes) {
    if (failed || !p) return nullptr;
    if (is_device_ptr(p)) return p;
    any_host = true;
    const void *d = resident(p, bytes);
    if (!d) failed = true;
    return d;
}

int CallScope::finish() {
    cudaStream_t s = stream();
    if (failed) {
        if (s) cudaStreamSynchronize(s);
        return mlq_last_error() ? mlq_last_error() : MLQ_ERR_CUDA;
    }
    for (int i = 0; i < n_pending_; i++) {
        if (!MLQ_CUDA(cudaMemcpyAsync(pending_[i].host, pending_[i].dev, pending_[i].bytes,
                                      cudaMemcpyDeviceToHost, s)))
            return MLQ_ERR_CUDA;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(MLQ_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
        return MLQ_ERR_CUDA;
    }
    if (any_host) {
        if (!MLQ_CUDA(cudaStreamSynchronize(s))) return MLQ_ERR_CUDA;
        // the call waited for its kernels anyway: report a bounded wait that gave up
        if (Ctx *c = ctx()) return take_device_status(c);
    }
    return MLQ_OK;
}

}  // namespace mlq

// ====================================================================================== C-ABI
using namespace mlq;

extern "C" {

int mlq_last_error(void) { return t_err; }
const char *mlq_last_error_message(void) { return t_msg; }
void mlq_clear_error(void) { t_err = MLQ_OK; t_msg[0] = 0; }

int mlq_init(int device) {
    t_dev = device;
    return ctx() ? MLQ_OK : mlq_last_error();
}

int mlq_set_device(int device) { return mlq_init(device); }
int mlq_get_device(void) { return t_dev < 0 ? 0 : t_dev; }

void *mlq_get_stream(void) { return (void *)stream(); }

int mlq_set_stream(void *s) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    cudaStream_t ns = (cudaStream_t)s;   // 0 = the legacy default stream, as in CUDA
    if (ns != c->stream) cudaStreamSynchronize(c->stream);   // keep the arena's stream ordering
    c->stream = ns;
    return MLQ_OK;
}

int mlq_use_own_stream(void) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    if (c->stream != c->own_stream) cudaStreamSynchronize(c->stream);
    c->stream = c->own_stream;
    return MLQ_OK;
}

int mlq_device_status(void) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    if (!MLQ_CUDA(cudaStreamSynchronize(c->stream))) return MLQ_ERR_CUDA;
    return take_device_status(c);
}

// Self-test of the bounded-wait error path: one thread waits on a shared-memory mbarrier
// that nothing ever arrives on, gives up after limit_us microseconds of %globaltimer and
// writes DEV_ST_WAIT_FULL to the status word -- the path every pipeline wait of the
// library takes when its producer never delivers.  Nothing faults or hangs.
__global__ void k_wait_selftest(int *status, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (!mbar_wait_bounded(&bar, 0, limit_ns)) report_status(status, DEV_ST_WAIT_FULL);
}

int mlq_selftest_wait_timeout(int limit_us) {
    if (limit_us <= 0 || limit_us > 1000000) {
        set_error(MLQ_ERR_ARG, "mlq_selftest_wait_timeout: limit %d us outside 1..1000000", limit_us);
        return MLQ_ERR_ARG;
    }
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    k_wait_selftest<<<1, 32, 0, c->stream>>>(c->d_status, 1000ull * (unsigned long long)limit_us);
    count_launch();
    if (!MLQ_CUDA(cudaGetLastError())) return MLQ_ERR_CUDA;
    return mlq_sync();
}

int mlq_sync(void) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    if (!MLQ_CUDA(cudaStreamSynchronize(c->stream))) return MLQ_ERR_CUDA;
    return mlq_device_status();
}

// Upload a whole host tensor once; every pointer inside [p, p + bytes) then resolves to
// its device copy without a content check (the caller promises the bytes stay fixed).
int mlq_register_weights(const void *p, size_t bytes) {
    if (!p || !bytes) { set_error(MLQ_ERR_ARG, "register_weights: null/empty"); return MLQ_ERR_ARG; }
    if (is_device_ptr(p)) return MLQ_OK;
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    std::lock_guard<std::mutex> lk(g_mu);
    if (in_registered_range(c->device, p, bytes)) return MLQ_OK;
    void *d = nullptr;
    if (!MLQ_CUDA(cudaMalloc(&d, bytes + 256))) return MLQ_ERR_CUDA;
    if (!MLQ_CUDA(cudaMemcpy(d, p, bytes, cudaMemcpyHostToDevice))) { cudaFree(d); return MLQ_ERR_CUDA; }
    cudaMemset((char *)d + bytes, 0, 256);
    RangeEntry e{bytes, d, {}};
    range_sample((const uint8_t *)p, bytes, e.sample);
    g_ranges[c->device][(uintptr_t)p] = std::move(e);
    g_cache_bytes[c->device] += bytes;
    return MLQ_OK;
}

// Drop the device copy of a tensor registered at exactly `p` (call before freeing it).
int mlq_unregister_weights(const void *p) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    cudaStreamSynchronize(c->stream);
    std::lock_guard<std::mutex> lk(g_mu);
    auto &m = g_ranges[c->device];
    auto it = m.find((uintptr_t)p);
    if (it == m.end()) {
        set_error(MLQ_ERR_ARG, "unregister_weights: %p was not registered", p);
        return MLQ_ERR_ARG;
    }
    cudaFree(it->second.dev);
    g_cache_bytes[c->device] -= it->second.bytes;
    m.erase(it);
    return MLQ_OK;
}

int mlq_cache_clear(void) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    mlq_forget_model_plans();
    forget_kv_mirrors();
    forget_tc_scratch();
    cudaStreamSynchronize(c->stream);
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto &kv : g_cache[c->device]) cudaFree(kv.second.dev);
    g_cache[c->device].clear();
    for (auto &kv : g_ranges[c->device]) cudaFree(kv.second.dev);
    g_ranges[c->device].clear();
    g_cache_bytes[c->device] = 0;
    return MLQ_OK;
}

size_t mlq_cache_bytes(void) {
    Ctx *c = ctx();
    return c ? g_cache_bytes[c->device] : 0;
}

int mlq_num_sms(void) {
    Ctx *c = ctx();
    return c ? c->num_sms : 0;
}

unsigned long long mlq_launch_count(void) { return g_launches.load(); }

int mlq_set_ref_compat(int on) {
    g_compat.store(on ? 1 : 0);
    return MLQ_OK;
}
int mlq_get_ref_compat(void) { return ref_compat() ? 1 : 0; }

}  // extern "C"
