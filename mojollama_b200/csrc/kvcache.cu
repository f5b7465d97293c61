// PagedAttention bookkeeping of the reference (cengine_batch_instr.c:160-214) with the
// same structs, byte for byte, so ctypes mirrors (forward/zaya_bc.py:32-130 of the
// reference) keep working:
//   PageTable { page_size, n_pages, pages, table, free_pages, free_count, _nkh, _hd, _n_layers }
//   KVBlock   { k, v, n_blocks, seq_len[64], block_map[64][1024], pt }
// Difference: `pages`, `k` and `v` are device memory (HBM) here -- the KV cache lives
// where attention runs; `table` and `free_pages` stay host memory (pure bookkeeping,
// uploaded with each step).  The page pool is [n_layers][n_pages][page_size][nkh*hd]
// for K followed by the same for V (cengine_batch_instr.c:1354-1361).
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "mlq_internal.h"

namespace mlq {
constexpr int kMaxBlocks = 1024;   // MAX_BLOCKS, cengine_batch_instr.c:23
constexpr int kBlockSize = 64;     // BLOCK_SIZE, cengine_batch_instr.c:22

// sizes of the k/v arrays kv_init allocated, so a kernel writing them can check its extent
static std::mutex g_kv_mu;
static std::map<const void *, size_t> g_kv_arrays;

size_t kv_array_bytes(const void *p) {
    std::lock_guard<std::mutex> lk(g_kv_mu);
    auto it = g_kv_arrays.find(p);
    return it == g_kv_arrays.end() ? 0 : it->second;
}
}  // namespace mlq

using namespace mlq;

extern "C" {

int mlq_page_table_init(MlqPageTable *pt, int max_pages, int page_size, int nkh, int hd, int n_layers) {
    if (!pt || max_pages <= 0 || page_size <= 0 || nkh <= 0 || hd <= 0 || n_layers <= 0) {
        set_error(MLQ_ERR_ARG, "page_table_init: bad arguments");
        return MLQ_ERR_ARG;
    }
    if (!ctx()) return mlq_last_error();
    memset(pt, 0, sizeof(*pt));
    pt->page_size = page_size;
    pt->n_pages = max_pages;
    pt->_nkh = nkh;
    pt->_hd = hd;
    pt->_n_layers = n_layers;
    const size_t total = (size_t)n_layers * max_pages * page_size * nkh * hd * 2;
    void *d = nullptr;
    if (!MLQ_CUDA(cudaMalloc(&d, total * sizeof(float)))) return MLQ_ERR_CUDA;
    if (!MLQ_CUDA(cudaMemset(d, 0, total * sizeof(float)))) { cudaFree(d); return MLQ_ERR_CUDA; }
    pt->pages = (float *)d;
    pt->table = (int *)malloc(kMaxBlocks * sizeof(int));
    pt->free_pages = (int *)malloc((size_t)max_pages * sizeof(int));
    if (!pt->table || !pt->free_pages) {
        set_error(MLQ_ERR_CAPACITY, "page_table_init: host allocation failed");
        return MLQ_ERR_CAPACITY;
    }
    memset(pt->table, -1, kMaxBlocks * sizeof(int));
    for (int i = 0; i < max_pages; i++) pt->free_pages[i] = max_pages - 1 - i;   // LIFO: page 0 first
    pt->free_count = max_pages;
    return MLQ_OK;
}

int mlq_page_table_alloc(MlqPageTable *pt) {
    if (!pt || pt->free_count <= 0) return -1;
    return pt->free_pages[--pt->free_count];
}

void mlq_page_table_free(MlqPageTable *pt, int page_id) {
    if (pt && pt->free_count < pt->n_pages) pt->free_pages[pt->free_count++] = page_id;
}

void mlq_map_page(MlqPageTable *pt, int logical_page, int physical_page) {
    if (pt && logical_page >= 0 && logical_page < kMaxBlocks) pt->table[logical_page] = physical_page;
}

void mlq_page_table_destroy(MlqPageTable *pt) {
    if (!pt) return;
    if (pt->pages) cudaFree(pt->pages);
    free(pt->table);
    free(pt->free_pages);
    memset(pt, 0, sizeof(*pt));
}

// kv_init (cengine_batch_instr.c:208): flat k/v of L * MAX_BLOCKS * BLOCK_SIZE * nkh * hd
// floats each plus a page table of MAX_BLOCKS pages of BLOCK_SIZE slots
int mlq_kv_init(MlqKVBlock *kv, int L, int nkh, int hd) {
    if (!kv || L <= 0 || nkh <= 0 || hd <= 0) {
        set_error(MLQ_ERR_ARG, "kv_init: bad arguments");
        return MLQ_ERR_ARG;
    }
    if (!ctx()) return mlq_last_error();
    const size_t sz = (size_t)L * kMaxBlocks * kBlockSize * nkh * hd * sizeof(float);
    void *k = nullptr, *v = nullptr;
    if (!MLQ_CUDA(cudaMalloc(&k, sz))) return MLQ_ERR_CUDA;
    if (!MLQ_CUDA(cudaMalloc(&v, sz))) { cudaFree(k); return MLQ_ERR_CUDA; }
    cudaMemset(k, 0, sz);
    cudaMemset(v, 0, sz);
    kv->k = (float *)k;
    kv->v = (float *)v;
    {
        std::lock_guard<std::mutex> lk(g_kv_mu);
        g_kv_arrays[k] = sz;
        g_kv_arrays[v] = sz;
    }
    kv->n_blocks = 0;
    memset(kv->block_map, -1, sizeof(kv->block_map));
    memset(kv->seq_len, 0, sizeof(kv->seq_len));
    return mlq_page_table_init(&kv->pt, kMaxBlocks, kBlockSize, nkh, hd, L);
}

int mlq_kv_alloc(MlqKVBlock *kv) { return kv ? mlq_page_table_alloc(&kv->pt) : -1; }

void mlq_kv_free(MlqKVBlock *kv) {
    if (!kv) return;
    {
        std::lock_guard<std::mutex> lk(g_kv_mu);
        g_kv_arrays.erase(kv->k);
        g_kv_arrays.erase(kv->v);
    }
    if (kv->k) cudaFree(kv->k);
    if (kv->v) cudaFree(kv->v);
    kv->k = kv->v = nullptr;
    mlq_page_table_destroy(&kv->pt);
}

// ------------------------------------------------------------------ snapshots (prefix cache)
// packed [2][L][len][row]: K of every layer, then V; element (kind, layer, pos, i) lives in
// the pool at ((kind * L + layer) * n_pages + table[pos / ps]) * ps + pos % ps, row i
__global__ void k_kv_pack(float *__restrict__ pool, const int *__restrict__ table, float *__restrict__ packed,
                          int L, int n_pages, int ps, int row, int len, int to_pool) {
    const int layer = blockIdx.y, kind = blockIdx.z;
    const long long n = (long long)len * row;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
        const int pos = (int)(e / row), i = (int)(e - (long long)pos * row);
        const long long slot = ((long long)(kind * L + layer) * n_pages + table[pos / ps]) * ps + pos % ps;
        float *pp = pool + slot * row + i;
        float *qq = packed + ((long long)(kind * L + layer) * len + pos) * row + i;
        if (to_pool) *pp = *qq;
        else *qq = *pp;
    }
}

static int kv_pack(MlqKVBlock *kv, int len, float *packed, int to_pool, const char *who) {
    const MlqPageTable &pt = kv->pt;
    const int row = pt._nkh * pt._hd, L = pt._n_layers;
    const int used = (len + pt.page_size - 1) / pt.page_size;
    for (int i = 0; i < used; i++) {
        if (pt.table[i] < 0 || pt.table[i] >= pt.n_pages) {
            set_error(MLQ_ERR_ARG, "%s: logical page %d unmapped or outside the pool (%d)", who, i, pt.table[i]);
            return MLQ_ERR_ARG;
        }
    }
    if (len == 0) return MLQ_OK;
    CallScope cs;
    const int *dt = (const int *)cs.in(pt.table, sizeof(int) * (size_t)used);
    float *dp = to_pool ? (float *)cs.in(packed, sizeof(float) * 2 * (size_t)L * len * row)
                        : (float *)cs.out(packed, sizeof(float) * 2 * (size_t)L * len * row);
    if (cs.failed) return cs.finish();
    const long long n = (long long)len * row;
    const unsigned gx = (unsigned)std::min<long long>((n + 255) / 256, 1024);
    k_kv_pack<<<dim3(gx, L, 2), 256, 0, stream()>>>(pt.pages, dt, dp, L, pt.n_pages, pt.page_size, row, len, to_pool);
    count_launch();
    if (!MLQ_CUDA(cudaGetLastError())) { cs.failed = true; cs.finish(); return MLQ_ERR_CUDA; }
    return cs.finish();
}

// Positions [0, len) of every layer's K and V rows out of a KVBlock's page pool, packed as
// [2][L][len][nkh*hd] floats at dst (device or host), following its page table.
int mlq_kv_snapshot(const MlqKVBlock *kv, int len, float *dst) {
    if (!kv || !dst || len < 0 || !kv->pt.pages || !kv->pt.table || len > kv->seq_len[0] ||
        len > kMaxBlocks * kv->pt.page_size) {
        set_error(MLQ_ERR_ARG, "mlq_kv_snapshot: bad block, destination or length (len <= seq_len)");
        return MLQ_ERR_ARG;
    }
    return kv_pack(const_cast<MlqKVBlock *>(kv), len, dst, 0, "mlq_kv_snapshot");
}

// The reverse: maps a page (from the block's free list) to every logical page of [0, len)
// that has none, copies src [2][L][len][nkh*hd] into those positions and sets seq_len to
// len.  The block then continues at position len as if it had run those tokens itself.
int mlq_kv_restore(MlqKVBlock *kv, int len, const float *src) {
    if (!kv || !src || len < 0 || !kv->pt.pages || !kv->pt.table || len > kMaxBlocks * kv->pt.page_size) {
        set_error(MLQ_ERR_ARG, "mlq_kv_restore: bad block, source or length");
        return MLQ_ERR_ARG;
    }
    const int used = (len + kv->pt.page_size - 1) / kv->pt.page_size;
    for (int i = 0; i < used; i++) {
        if (kv->pt.table[i] < 0) {
            const int page = mlq_page_table_alloc(&kv->pt);
            if (page < 0) {
                set_error(MLQ_ERR_CAPACITY, "mlq_kv_restore: page pool full at logical page %d", i);
                return MLQ_ERR_CAPACITY;
            }
            kv->pt.table[i] = page;
        }
    }
    const int rc = kv_pack(kv, len, const_cast<float *>(src), 1, "mlq_kv_restore");
    if (rc == MLQ_OK) kv->seq_len[0] = len;
    return rc;
}

size_t mlq_sizeof_page_table(void) { return sizeof(MlqPageTable); }
size_t mlq_sizeof_kv_block(void) { return sizeof(MlqKVBlock); }

// kv_cache_update (simd_ops.c:209): copy one position's K/V rows (nkh*hd floats) to
// offset n_past*nkh*hd of flat caches; `layer` and `max_seq` are ignored, as there
int mlq_kv_cache_update(float *k_cache, float *v_cache, const float *k_new, const float *v_new, int layer,
                        int n_past, int max_seq, int nkh, int hd) {
    (void)layer;
    (void)max_seq;
    if (!k_cache || !v_cache || !k_new || !v_new || n_past < 0 || nkh <= 0 || hd <= 0) {
        set_error(MLQ_ERR_ARG, "kv_cache_update: bad arguments");
        return MLQ_ERR_ARG;
    }
    const size_t row = (size_t)nkh * hd;
    const size_t off = (size_t)n_past * row;
    if (!is_device_ptr(k_cache) && !is_device_ptr(k_new) && !is_device_ptr(v_cache) && !is_device_ptr(v_new)) {
        memcpy(k_cache + off, k_new, row * sizeof(float));    // all host: nothing for the GPU to do
        memcpy(v_cache + off, v_new, row * sizeof(float));
        return MLQ_OK;
    }
    cudaStream_t s = stream();
    if (!MLQ_CUDA(cudaMemcpyAsync(k_cache + off, k_new, row * sizeof(float), cudaMemcpyDefault, s))) return MLQ_ERR_CUDA;
    if (!MLQ_CUDA(cudaMemcpyAsync(v_cache + off, v_new, row * sizeof(float), cudaMemcpyDefault, s))) return MLQ_ERR_CUDA;
    return MLQ_CUDA(cudaStreamSynchronize(s)) ? MLQ_OK : MLQ_ERR_CUDA;
}

}  // extern "C"
