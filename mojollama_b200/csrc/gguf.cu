// GGUF reader and device weight loader: mmap -> pinned staging -> HBM.
//
// The reference parses GGUF files with gguf-py's GGUFReader (un-pinned in the reference,
// 0.19.0 here) and keeps every quantized tensor as a numpy view of the mmapped file, or
// dequantises it to F32 on the host (src/mojollama/kernels/turbo_engine_v7_moe.py:425-618);
// the C engine then reads those host buffers.  Here the file is parsed natively and its
// data section goes to HBM unchanged, GGUF blocks in their byte layout, in one streaming
// pass: a pool of host threads copies consecutive chunks of the mapped file into two pinned
// buffers while the copy engine moves the previous chunk to the device.  A tensor's device
// address is then the upload base plus its offset inside the data section; small tensors
// can be turned into F32 on the device with mlq_dequantize.
//
// Format (the public GGUF specification, versions 2 and 3; little-endian): magic "GGUF",
// u32 version, u64 tensor count, u64 metadata count; metadata pairs (string key, u32 value
// type, value: u8 i8 u16 i16 u32 i32 f32 bool string array u64 i64 f64 for types 0..12,
// an array being u32 item type + u64 count + items); tensor infos (string name, u32 n_dims,
// u64 dims[n_dims] fastest first, u32 ggml type, u64 offset inside the data section); the
// data section starts at the next multiple of general.alignment (default 32).  A string is
// u64 length + bytes.  Parsing checks every length against the file size.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "mlq_internal.h"

namespace mlq {

// (elements, bytes) per block of the ggml types whose layout is fixed (the GGUF
// specification's type table; checked against gguf-py's GGML_QUANT_SIZES in the tests)
static bool ggml_block(int t, int &be, int &bb) {
    switch (t) {
        case 0: be = 1; bb = 4; return true;      // F32
        case 1: be = 1; bb = 2; return true;      // F16
        case 2: be = 32; bb = 18; return true;    // Q4_0
        case 3: be = 32; bb = 20; return true;    // Q4_1
        case 6: be = 32; bb = 22; return true;    // Q5_0
        case 7: be = 32; bb = 24; return true;    // Q5_1
        case 8: be = 32; bb = 34; return true;    // Q8_0
        case 9: be = 32; bb = 40; return true;    // Q8_1
        case 10: be = 256; bb = 84; return true;  // Q2_K
        case 11: be = 256; bb = 110; return true; // Q3_K
        case 12: be = 256; bb = 144; return true; // Q4_K
        case 13: be = 256; bb = 176; return true; // Q5_K
        case 14: be = 256; bb = 210; return true; // Q6_K
        case 15: be = 256; bb = 292; return true; // Q8_K
        case 24: be = 1; bb = 1; return true;     // I8
        case 25: be = 1; bb = 2; return true;     // I16
        case 26: be = 1; bb = 4; return true;     // I32
        case 27: be = 1; bb = 8; return true;     // I64
        case 28: be = 1; bb = 8; return true;     // F64
        case 30: be = 1; bb = 2; return true;     // BF16
        case 39: be = 32; bb = 17; return true;   // MXFP4
        default: return false;
    }
}

struct GgufTensor {
    std::string name;
    int n_dims = 0;
    int64_t dims[4] = {1, 1, 1, 1};
    int type = 0;
    uint64_t offset = 0;   // inside the data section
    uint64_t bytes = 0;    // 0 when the type's layout is not known here
};

struct GgufKV {
    int type = 0;          // value type (9 = array)
    int item_type = 0;     // arrays
    uint64_t count = 0;    // arrays
    size_t pos = 0;        // file offset of the value (of the first item for arrays)
};

struct GgufFile {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    uint64_t alignment = 32;
    size_t data_off = 0;
    std::vector<GgufTensor> tensors;
    std::map<std::string, GgufKV> kv;
    std::map<std::string, size_t> by_name;
};

struct Cursor {
    const uint8_t *p;
    size_t size, pos = 0;
    bool ok = true;
    bool need(size_t n) {
        if (!ok || n > size - pos) ok = false;
        return ok;
    }
    template <typename T> T get() {
        T v{};
        if (need(sizeof(T))) { memcpy(&v, p + pos, sizeof(T)); pos += sizeof(T); }
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!need(n)) return std::string();
        std::string s((const char *)p + pos, (size_t)n);
        pos += n;
        return s;
    }
    void skip_str() {
        const uint64_t n = get<uint64_t>();
        if (need(n)) pos += n;
    }
};

static size_t scalar_size(int t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

static void skip_value(Cursor &c, int t, int depth = 0) {
    if (depth > 4) { c.ok = false; return; }
    if (t == 8) { c.skip_str(); return; }
    if (t == 9) {
        const int it = (int)c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        if (it == 8 || it == 9) {
            for (uint64_t i = 0; i < n && c.ok; i++) skip_value(c, it, depth + 1);
        } else {
            const size_t sz = scalar_size(it);
            if (!sz || n > (c.size - c.pos) / sz) { c.ok = false; return; }
            c.pos += (size_t)n * sz;
        }
        return;
    }
    const size_t sz = scalar_size(t);
    if (!sz || !c.need(sz)) { c.ok = false; return; }
    c.pos += sz;
}

static bool parse(GgufFile &f, char *why, size_t why_len) {
    Cursor c{f.map, f.size};
    const uint32_t magic = c.get<uint32_t>();
    if (!c.ok || magic != 0x46554747u) { snprintf(why, why_len, "not a GGUF file (magic)"); return false; }
    f.version = c.get<uint32_t>();
    if (f.version != 2 && f.version != 3) { snprintf(why, why_len, "GGUF version %u not supported (2, 3)", f.version); return false; }
    const uint64_t n_t = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
    if (!c.ok || n_t > (1u << 24) || n_kv > (1u << 24)) { snprintf(why, why_len, "implausible counts"); return false; }
    for (uint64_t i = 0; i < n_kv && c.ok; i++) {
        std::string key = c.str();
        GgufKV v;
        v.type = (int)c.get<uint32_t>();
        if (v.type == 9) {
            const size_t at = c.pos;
            v.item_type = (int)c.get<uint32_t>();
            v.count = c.get<uint64_t>();
            v.pos = c.pos;
            c.pos = at;
        } else {
            v.pos = c.pos;
        }
        skip_value(c, v.type);
        if (c.ok) f.kv[key] = v;
    }
    if (!c.ok) { snprintf(why, why_len, "truncated metadata"); return false; }
    auto al = f.kv.find("general.alignment");
    if (al != f.kv.end() && al->second.type == 4) {
        uint32_t a;
        memcpy(&a, f.map + al->second.pos, 4);
        if (a == 0 || (a & (a - 1))) { snprintf(why, why_len, "alignment %u not a power of two", a); return false; }
        f.alignment = a;
    }
    f.tensors.resize((size_t)n_t);
    for (uint64_t i = 0; i < n_t && c.ok; i++) {
        GgufTensor &t = f.tensors[(size_t)i];
        t.name = c.str();
        t.n_dims = (int)c.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) { c.ok = false; break; }
        for (int d = 0; d < t.n_dims; d++) {
            const uint64_t v = c.get<uint64_t>();
            if (v == 0 || v > ((uint64_t)1 << 40)) { c.ok = false; break; }
            t.dims[d] = (int64_t)v;
        }
        if (!c.ok) break;
        t.type = (int)c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        int be = 0, bb = 0;
        if (ggml_block(t.type, be, bb) && t.dims[0] % be == 0) {
            // dims are <= 2^40 each; the product of the outer ones is checked against the file
            unsigned __int128 n = 1;
            for (int d = 1; d < t.n_dims; d++) n *= (uint64_t)t.dims[d];
            n *= (unsigned __int128)(t.dims[0] / be) * bb;
            if (n > (unsigned __int128)f.size) { c.ok = false; break; }
            t.bytes = (uint64_t)n;
        }
        f.by_name[t.name] = (size_t)i;
    }
    if (!c.ok) { snprintf(why, why_len, "truncated tensor infos"); return false; }
    f.data_off = (c.pos + f.alignment - 1) / f.alignment * f.alignment;
    if (f.data_off > f.size) { snprintf(why, why_len, "data section beyond the file"); return false; }
    for (auto &t : f.tensors) {
        const uint64_t avail = f.size - f.data_off;
        if (t.offset % f.alignment || t.offset > avail || t.bytes > avail - t.offset) {
            snprintf(why, why_len, "tensor %s at %llu (+%llu bytes) outside the data section", t.name.c_str(),
                     (unsigned long long)t.offset, (unsigned long long)t.bytes);
            return false;
        }
    }
    return true;
}

// ------------------------------------------------------------------ streaming upload
constexpr size_t kStageBytes = (size_t)64 << 20;   // per pinned buffer

struct Stage {
    uint8_t *buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    bool ready = false;
};
static Stage g_stage[16];
static std::mutex g_stage_mu;

static bool stage_for(int dev, Stage *&st) {
    st = &g_stage[dev];
    if (st->ready) return true;
    for (int i = 0; i < 2; i++) {
        if (!MLQ_CUDA(cudaHostAlloc((void **)&st->buf[i], kStageBytes, cudaHostAllocPortable))) return false;
        if (!MLQ_CUDA(cudaEventCreateWithFlags(&st->done[i], cudaEventDisableTiming))) return false;
    }
    st->ready = true;
    return true;
}

static void parallel_copy(uint8_t *dst, const uint8_t *src, size_t n, int threads) {
    if (threads <= 1 || n < ((size_t)4 << 20)) {
        memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> pool;
    const size_t per = (n / threads + 4095) & ~(size_t)4095;
    for (int i = 0; i < threads; i++) {
        const size_t a = (size_t)i * per;
        if (a >= n) break;
        const size_t len = std::min(per, n - a);
        pool.emplace_back([=] { memcpy(dst + a, src + a, len); });
    }
    for (auto &t : pool) t.join();
}

// file bytes [off, off + n) -> dev, through the pinned double buffer on stream s
static int upload_range(const GgufFile &f, size_t off, size_t n, uint8_t *dev, cudaStream_t s) {
    Ctx *c = ctx();
    if (!c) return mlq_last_error();
    std::lock_guard<std::mutex> lk(g_stage_mu);
    Stage *st = nullptr;
    if (!stage_for(c->device, st)) return MLQ_ERR_CUDA;
    unsigned hw = std::thread::hardware_concurrency();
    const int threads = (int)std::min(8u, std::max(1u, hw / 2));
    madvise((void *)((uintptr_t)(f.map + off) & ~(uintptr_t)4095), n + 4096, MADV_SEQUENTIAL);
    size_t done = 0;
    int i = 0;
    while (done < n) {
        const int k = i & 1;
        const size_t len = std::min(kStageBytes, n - done);
        if (!MLQ_CUDA(cudaEventSynchronize(st->done[k]))) return MLQ_ERR_CUDA;   // buffer k free again
        parallel_copy(st->buf[k], f.map + off + done, len, threads);
        if (!MLQ_CUDA(cudaMemcpyAsync(dev + done, st->buf[k], len, cudaMemcpyHostToDevice, s))) return MLQ_ERR_CUDA;
        if (!MLQ_CUDA(cudaEventRecord(st->done[k], s))) return MLQ_ERR_CUDA;
        done += len;
        i++;
    }
    return MLQ_CUDA(cudaStreamSynchronize(s)) ? MLQ_OK : MLQ_ERR_CUDA;
}

}  // namespace mlq

using namespace mlq;

extern "C" {

void *mlq_gguf_open(const char *path) {
    if (!path) { set_error(MLQ_ERR_ARG, "mlq_gguf_open: null path"); return nullptr; }
    const int fd = open(path, O_RDONLY);
    if (fd < 0) { set_error(MLQ_ERR_ARG, "mlq_gguf_open: cannot open %s", path); return nullptr; }
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 24) {
        close(fd);
        set_error(MLQ_ERR_ARG, "mlq_gguf_open: %s is too short for a GGUF header", path);
        return nullptr;
    }
    void *m = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        close(fd);
        set_error(MLQ_ERR_ARG, "mlq_gguf_open: mmap of %s failed", path);
        return nullptr;
    }
    GgufFile *f = new GgufFile;
    f->fd = fd;
    f->map = (const uint8_t *)m;
    f->size = (size_t)sb.st_size;
    char why[256] = {0};
    if (!parse(*f, why, sizeof why)) {
        munmap((void *)f->map, f->size);
        close(fd);
        delete f;
        set_error(MLQ_ERR_ARG, "mlq_gguf_open: %s: %s", path, why);
        return nullptr;
    }
    return f;
}

int mlq_gguf_close(void *h) {
    GgufFile *f = static_cast<GgufFile *>(h);
    if (!f) return MLQ_ERR_ARG;
    munmap((void *)f->map, f->size);
    close(f->fd);
    delete f;
    return MLQ_OK;
}

int mlq_gguf_version(void *h) { return h ? (int)static_cast<GgufFile *>(h)->version : -1; }
int64_t mlq_gguf_n_tensors(void *h) { return h ? (int64_t)static_cast<GgufFile *>(h)->tensors.size() : -1; }
int64_t mlq_gguf_n_kv(void *h) { return h ? (int64_t)static_cast<GgufFile *>(h)->kv.size() : -1; }
uint64_t mlq_gguf_data_offset(void *h) { return h ? static_cast<GgufFile *>(h)->data_off : 0; }
uint64_t mlq_gguf_data_bytes(void *h) {
    if (!h) return 0;
    const GgufFile *f = static_cast<GgufFile *>(h);
    return f->size - f->data_off;
}
uint64_t mlq_gguf_alignment(void *h) { return h ? static_cast<GgufFile *>(h)->alignment : 0; }

int mlq_gguf_tensor(void *h, int64_t i, MlqGgufTensor *out) {
    const GgufFile *f = static_cast<GgufFile *>(h);
    if (!f || !out || i < 0 || i >= (int64_t)f->tensors.size()) {
        set_error(MLQ_ERR_ARG, "mlq_gguf_tensor: bad handle or index");
        return MLQ_ERR_ARG;
    }
    const GgufTensor &t = f->tensors[(size_t)i];
    memset(out, 0, sizeof(*out));
    snprintf(out->name, sizeof(out->name), "%s", t.name.c_str());
    out->n_dims = t.n_dims;
    for (int d = 0; d < 4; d++) out->dims[d] = t.dims[d];
    out->type = t.type;
    out->offset = t.offset;
    out->bytes = t.bytes;
    return MLQ_OK;
}

int64_t mlq_gguf_find(void *h, const char *name) {
    const GgufFile *f = static_cast<GgufFile *>(h);
    if (!f || !name) return -1;
    auto it = f->by_name.find(name);
    return it == f->by_name.end() ? -1 : (int64_t)it->second;
}

static const GgufKV *find_kv(void *h, const char *key) {
    const GgufFile *f = static_cast<GgufFile *>(h);
    if (!f || !key) return nullptr;
    auto it = f->kv.find(key);
    return it == f->kv.end() ? nullptr : &it->second;
}

// metadata value type of `key` (0..12), -1 if absent
int mlq_gguf_kv_type(void *h, const char *key) {
    const GgufKV *v = find_kv(h, key);
    return v ? v->type : -1;
}

int mlq_gguf_kv_int(void *h, const char *key, int64_t *out) {
    const GgufKV *v = find_kv(h, key);
    if (!v || !out) { set_error(MLQ_ERR_ARG, "mlq_gguf_kv_int: no key %s", key ? key : "(null)"); return MLQ_ERR_ARG; }
    const uint8_t *p = static_cast<GgufFile *>(h)->map + v->pos;
    switch (v->type) {
        case 0: *out = *(const uint8_t *)p; return MLQ_OK;
        case 1: *out = *(const int8_t *)p; return MLQ_OK;
        case 2: { uint16_t x; memcpy(&x, p, 2); *out = x; return MLQ_OK; }
        case 3: { int16_t x; memcpy(&x, p, 2); *out = x; return MLQ_OK; }
        case 4: { uint32_t x; memcpy(&x, p, 4); *out = x; return MLQ_OK; }
        case 5: { int32_t x; memcpy(&x, p, 4); *out = x; return MLQ_OK; }
        case 7: *out = *p ? 1 : 0; return MLQ_OK;
        case 10: { uint64_t x; memcpy(&x, p, 8); *out = (int64_t)x; return MLQ_OK; }
        case 11: { int64_t x; memcpy(&x, p, 8); *out = x; return MLQ_OK; }
        default: set_error(MLQ_ERR_TYPE, "mlq_gguf_kv_int: %s has value type %d", key, v->type); return MLQ_ERR_TYPE;
    }
}

int mlq_gguf_kv_float(void *h, const char *key, double *out) {
    const GgufKV *v = find_kv(h, key);
    if (!v || !out) { set_error(MLQ_ERR_ARG, "mlq_gguf_kv_float: no key %s", key ? key : "(null)"); return MLQ_ERR_ARG; }
    const uint8_t *p = static_cast<GgufFile *>(h)->map + v->pos;
    if (v->type == 6) { float x; memcpy(&x, p, 4); *out = x; return MLQ_OK; }
    if (v->type == 12) { double x; memcpy(&x, p, 8); *out = x; return MLQ_OK; }
    int64_t i = 0;
    if (mlq_gguf_kv_int(h, key, &i) == MLQ_OK) { *out = (double)i; return MLQ_OK; }
    set_error(MLQ_ERR_TYPE, "mlq_gguf_kv_float: %s has value type %d", key, v->type);
    return MLQ_ERR_TYPE;
}

// string value (NUL-terminated, truncated to len - 1); returns the full length, or -1
int64_t mlq_gguf_kv_str(void *h, const char *key, char *buf, size_t len) {
    const GgufKV *v = find_kv(h, key);
    if (!v || v->type != 8) { set_error(MLQ_ERR_ARG, "mlq_gguf_kv_str: no string key %s", key ? key : "(null)"); return -1; }
    const uint8_t *p = static_cast<GgufFile *>(h)->map + v->pos;
    uint64_t n;
    memcpy(&n, p, 8);
    if (buf && len) {
        const size_t k = (size_t)std::min<uint64_t>(n, len - 1);
        memcpy(buf, p + 8, k);
        buf[k] = 0;
    }
    return (int64_t)n;
}

// array metadata: item type and count (-1 when `key` is not an array)
int64_t mlq_gguf_kv_array(void *h, const char *key, int *item_type) {
    const GgufKV *v = find_kv(h, key);
    if (!v || v->type != 9) return -1;
    if (item_type) *item_type = v->item_type;
    return (int64_t)v->count;
}

// The whole data section (mlq_gguf_data_bytes bytes) into device memory at dev: tensor i
// then starts at dev + its offset.  Synchronous; streams the mapped file through two
// pinned buffers on the library stream.
int mlq_gguf_upload(void *h, void *dev, uint64_t dev_bytes) {
    const GgufFile *f = static_cast<GgufFile *>(h);
    if (!f || !dev) { set_error(MLQ_ERR_ARG, "mlq_gguf_upload: null handle or destination"); return MLQ_ERR_ARG; }
    const uint64_t n = f->size - f->data_off;
    if (dev_bytes < n) {
        set_error(MLQ_ERR_CAPACITY, "mlq_gguf_upload: destination %llu bytes < data section %llu",
                  (unsigned long long)dev_bytes, (unsigned long long)n);
        return MLQ_ERR_CAPACITY;
    }
    if (!is_device_ptr(dev)) { set_error(MLQ_ERR_ARG, "mlq_gguf_upload: destination is not device memory"); return MLQ_ERR_ARG; }
    return upload_range(*f, f->data_off, (size_t)n, (uint8_t *)dev, stream());
}

// One tensor's bytes into device memory at dev (dev_bytes >= its size).
int mlq_gguf_upload_tensor(void *h, int64_t i, void *dev, uint64_t dev_bytes) {
    const GgufFile *f = static_cast<GgufFile *>(h);
    if (!f || !dev || i < 0 || i >= (int64_t)f->tensors.size()) {
        set_error(MLQ_ERR_ARG, "mlq_gguf_upload_tensor: bad handle, index or destination");
        return MLQ_ERR_ARG;
    }
    const GgufTensor &t = f->tensors[(size_t)i];
    if (!t.bytes) { set_error(MLQ_ERR_TYPE, "mlq_gguf_upload_tensor: %s has ggml type %d of unknown size", t.name.c_str(), t.type); return MLQ_ERR_TYPE; }
    if (dev_bytes < t.bytes) { set_error(MLQ_ERR_CAPACITY, "mlq_gguf_upload_tensor: destination too small for %s", t.name.c_str()); return MLQ_ERR_CAPACITY; }
    if (!is_device_ptr(dev)) { set_error(MLQ_ERR_ARG, "mlq_gguf_upload_tensor: destination is not device memory"); return MLQ_ERR_ARG; }
    return upload_range(*f, f->data_off + t.offset, (size_t)t.bytes, (uint8_t *)dev, stream());
}

// host view of tensor i inside the mapped file (valid until mlq_gguf_close), or NULL
const void *mlq_gguf_tensor_data(void *h, int64_t i) {
    const GgufFile *f = static_cast<GgufFile *>(h);
    if (!f || i < 0 || i >= (int64_t)f->tensors.size()) return nullptr;
    return f->map + f->data_off + f->tensors[(size_t)i].offset;
}

}  // extern "C"
