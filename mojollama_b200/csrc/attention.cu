// Decode attention (one new query per sequence) over a flat or paged fp32 KV cache.
//
// Replaces gqa_attention_decode (gqa_attention.c:93: per KV head, Q.K^T / sqrt(hd) by
// sgemm, softmax, P.V), the static gqa of cengine_batch_instr.c:141 and its paged
// gather (cengine_batch_instr.c:1354-1401), and attention_forward (simd_ops.c:159).
//
// KV addressing (KVView): slot t of a sequence lives in page table[t / page_size]
// (identity when there is no table) at row t % page_size; a row holds NKH*HD floats,
// K and V in separate regions:
//   flat cache  [seq][NKH*HD]                      page_size = huge, table = null
//   paged pool  [page][page_size][NKH*HD] per layer  (PageTable, cengine_batch_instr.c:160-214)
// The kernel reads pages in place through the table -- no gather copy.
//
// Split-K flash decode: CTA (split, kv head g x query-head part, sequence b) streams a
// contiguous chunk of positions in 32-position tiles through shared memory, computes the
// scores of its query heads (all NH/NKH that share g, or a part of them when the launcher
// splits them over CTAs), keeps an online softmax (running max / sum) per head and
// accumulates P.V in registers; it writes (max, sum, acc[HD]) per head and split.  k_attn_merge combines the splits with their log-sum-exp weights.  With one
// split the first kernel writes the output directly.  Optional sliding window: only
// the last `window` positions are attended (GPT-OSS alternate layers).
// Roofline: HBM-bound on the K and V rows read (2 * seq * NKH * HD * 4 bytes per
// sequence and layer).
#include <cuda_runtime.h>
#include <math.h>

#include "formats.cuh"
#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

__device__ __forceinline__ const float *kv_kbase(const KVView &kv, int b) {
    return kv.pool_seq ? kv.pool_seq[b] + (long long)kv.layer * kv.layer_stride : kv.k;
}
__device__ __forceinline__ const float *kv_vbase(const KVView &kv, int b) {
    return kv.pool_seq ? kv.pool_seq[b] + (long long)(kv.n_layers + kv.layer) * kv.layer_stride : kv.v;
}

// float offset of slot t of sequence b, or -1 when its page id lies outside a checked pool
__device__ __forceinline__ long long kv_offset(const KVView &kv, int b, int t) {
    if (!kv.table) return (long long)t * kv.row_stride;
    const int page = kv.table[(size_t)b * kv.table_stride + t / kv.page_size];
    if (kv.n_pages > 0 && (unsigned)page >= (unsigned)kv.n_pages) return -1;
    return (long long)page * kv.page_stride + (long long)(t % kv.page_size) * kv.row_stride;
}

constexpr int kTile = 32;          // positions per shared-memory tile
constexpr int kAttnThreads = 128;

// smem: q [rep][HD], K tile [kTile][HD+1], V tile [kTile][HD], p [rep][kTile], m / l / c
// [rep], and with a fused RoPE the new k / v rows of this CTA's KV head [2][HD]
template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const float *__restrict__ q, KVView kv,
                                                              const int *__restrict__ seq_lens, int seq_len_scalar,
                                                              int nh, int nkh, int window, float scale,
                                                              int chunk, float *__restrict__ out,
                                                              float *__restrict__ part_ml, float *__restrict__ part_acc,
                                                              uint8_t *__restrict__ planes, AttnRope rp) {
    extern __shared__ float sm[];
    pdl_wait();   // q, the KV rows and the split scratch follow earlier kernels
    pdl_trigger();
    // blockIdx.y = KV head g x query-head part hp: this CTA takes rep of the KV head's nh / nkh
    // query heads, from query head h0
    const int hsplit = gridDim.y / nkh;
    const int split = blockIdx.x, g = blockIdx.y / hsplit, hp = blockIdx.y - g * hsplit, b = blockIdx.z;
    const int rep = nh / nkh / hsplit;
    const int h0 = g * (nh / nkh) + hp * rep;
    const int n_splits = gridDim.x;
    const int sl = seq_lens ? seq_lens[b] : seq_len_scalar;
    const int lo_all = (window > 0 && sl > window) ? sl - window : 0;
    const int t0 = lo_all + split * chunk;
    const int t1 = min(sl, t0 + chunk);
    float *qs = sm;                                  // rep * HD
    float *ks = qs + rep * HD;                       // kTile * (HD + 1)
    float *vs = ks + kTile * (HD + 1);               // kTile * HD
    float *ps = vs + kTile * HD;                     // rep * kTile
    float *ms = ps + rep * kTile;                    // rep running max
    float *ls = ms + rep;                            // rep running sum
    float *cs = ls + rep;                            // rep correction factor of this tile
    float *nk = cs + rep;                            // fused RoPE: new k row of head g [HD]
    float *nv = nk + HD;                             //             new v row [HD]
    const int tid = threadIdx.x;
    const int p_new = rp.pos ? rp.pos[b] : -1;
    if (rp.pos) {
        // q heads g*rep.. and the new k row of head g, rotated as k_rope_kv does, then q scaled
        const int hd2 = rp.rope_dim / 2, row = nkh * HD;
        for (int i = tid; i < rep * HD; i += blockDim.x) qs[i] = q[((size_t)b * nh + (size_t)h0) * HD + i];
        for (int d = tid; d < HD; d += blockDim.x) {
            nk[d] = rp.k_new[(size_t)b * row + (size_t)g * HD + d];
            nv[d] = rp.v_new[(size_t)b * row + (size_t)g * HD + d];
        }
        __syncthreads();
        const float *cst = rp.cos_t + (size_t)p_new * hd2, *snt = rp.sin_t + (size_t)p_new * hd2;
        for (int t = tid; t < (rep + 1) * hd2; t += blockDim.x) {
            const int hh = t / hd2, j = t - hh * hd2;
            float *w = hh < rep ? qs + hh * HD : nk;
            const float c = cst[j], sv = snt[j];
            const float a0 = w[j], a1 = w[j + hd2];
            w[j] = a0 * c - a1 * sv;
            w[j + hd2] = a1 * c + a0 * sv;
        }
        __syncthreads();
        for (int i = tid; i < rep * HD; i += blockDim.x) qs[i] *= scale;
    } else {
        for (int i = tid; i < rep * HD; i += blockDim.x)
            qs[i] = q[((size_t)b * nh + (size_t)h0) * HD + i] * scale;
    }
    for (int h = tid; h < rep; h += blockDim.x) {
        ms[h] = -INFINITY;
        ls[h] = 0.0f;
    }
    // accumulators: thread owns (h, d) pairs tid, tid + 128, ...
    constexpr int kMaxAcc = 16;   // rep * HD <= 16 * 128
    float acc[kMaxAcc];
#pragma unroll
    for (int i = 0; i < kMaxAcc; i++) acc[i] = 0.0f;
    __syncthreads();

    const float *kb = kv_kbase(kv, b);
    const float *vb = kv_vbase(kv, b);
    if (rp.pos && hp == 0 && p_new >= t0 && p_new < t1) {
        // this CTA's positions include the new one (and it is head g's first part): store the
        // k / v rows of head g
        const long long off = kv_offset(kv, b, p_new);
        if (off >= 0) {
            const int row = nkh * HD;
            float *kc = const_cast<float *>(kb), *vc = const_cast<float *>(vb);
            float *mkb = rp.mk ? rp.mk[b] : nullptr, *mvb = rp.mv ? rp.mv[b] : nullptr;
            size_t moff = 0;
            bool mirror = mkb && mvb && kv.table;
            if (mirror) {
                const int page = kv.table[(size_t)b * kv.table_stride + p_new / kv.page_size];
                mirror = page >= 0 && page < 1024;
                moff = ((size_t)kv.layer * 1024 * 64 + (size_t)page * 64 + (p_new % kv.page_size)) * row;
            }
            for (int d = tid; d < HD; d += blockDim.x) {
                kc[off + (long long)g * HD + d] = nk[d];
                vc[off + (long long)g * HD + d] = nv[d];
                if (mirror) {
                    mkb[moff + (size_t)g * HD + d] = nk[d];
                    mvb[moff + (size_t)g * HD + d] = nv[d];
                }
            }
        }
    }
    for (int base = t0; base < t1; base += kTile) {
        const int nt = min(kTile, t1 - base);
        // stage K and V rows of this tile (coalesced along HD)
        for (int i = tid; i < nt * HD; i += blockDim.x) {
            const int t = i / HD, d = i - t * HD;
            if (base + t == p_new) {   // fused RoPE: the new row from shared memory
                ks[t * (HD + 1) + d] = nk[d];
                vs[t * HD + d] = nv[d];
                continue;
            }
            if (kv.tail_k && base + t == sl - 1) {
                const size_t o = (size_t)b * kv.tail_stride + (size_t)g * HD + d;
                ks[t * (HD + 1) + d] = kv.tail_k[o];
                vs[t * HD + d] = kv.tail_v[o];
                continue;
            }
            const long long slot = kv_offset(kv, b, base + t);
            if (slot < 0) {   // corrupt page id in a checked pool: zeros, no access
                ks[t * (HD + 1) + d] = 0.0f;
                vs[t * HD + d] = 0.0f;
                continue;
            }
            const long long off = slot + (long long)g * HD + d;
            ks[t * (HD + 1) + d] = kb[off];
            vs[t * HD + d] = vb[off];
        }
        __syncthreads();
        // scores p[h][t] = q_h . k_t (q already scaled)
        for (int i = tid; i < rep * kTile; i += blockDim.x) {
            const int h = i / kTile, t = i - h * kTile;
            float s = -INFINITY;
            if (t < nt) {
                s = 0.0f;
                const float *qh = qs + h * HD;
                const float *kt = ks + t * (HD + 1);
#pragma unroll 8
                for (int d = 0; d < HD; d++) s = fmaf(qh[d], kt[d], s);
            }
            ps[i] = s;
        }
        __syncthreads();
        // online softmax update per head (one warp per head)
        const int warp = tid >> 5, lane = tid & 31;
        for (int h = warp; h < rep; h += blockDim.x / 32) {
            const float s = ps[h * kTile + lane];
            float mx = s;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_old = ms[h];
            const float m_new = fmaxf(m_old, mx);
            const float e = (lane < nt) ? expf(s - m_new) : 0.0f;
            float sum = e;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            ps[h * kTile + lane] = e;
            if (lane == 0) {
                const float c = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
                cs[h] = c;
                ls[h] = ls[h] * c + sum;
                ms[h] = m_new;
            }
        }
        __syncthreads();
        // acc = acc * c + sum_t p[h][t] v[t][d]
#pragma unroll
        for (int j = 0; j < kMaxAcc; j++) {
            const int i = tid + j * kAttnThreads;
            if (i < rep * HD) {
                const int h = i / HD, d = i - h * HD;
                float a = acc[j] * cs[h];
                const float *ph = ps + h * kTile;
                for (int t = 0; t < nt; t++) a = fmaf(ph[t], vs[t * HD + d], a);
                acc[j] = a;
            }
        }
        __syncthreads();
    }
    // write the result (one split) or this split's partial state
#pragma unroll
    for (int j = 0; j < kMaxAcc; j++) {
        const int i = tid + j * kAttnThreads;
        if (i < rep * HD) {
            const int h = i / HD, d = i - h * HD;
            const int head = h0 + h;
            if (n_splits == 1) {
                const float l = ls[h];
                out[((size_t)b * nh + head) * HD + d] = (l > 0.0f) ? acc[j] / l : 0.0f;
            } else {
                part_acc[(((size_t)b * nh + head) * n_splits + split) * HD + d] = acc[j];
            }
        }
    }
    if (n_splits > 1) {
        for (int h = tid; h < rep; h += blockDim.x) {
            const size_t o = (((size_t)b * nh + h0 + h) * n_splits + split) * 2;
            part_ml[o] = ms[h];
            part_ml[o + 1] = ls[h];
        }
    } else if (planes) {
        // the output rows also as packed activation rows (the next GEMV's input encoding):
        // this CTA's rep heads are rep * HD / 32 whole 32-element blocks of row b
        __syncthreads();
        const int warp = tid >> 5, lane = tid & 31, K = nh * HD;
        const int kb0 = h0 * HD / 32;
        for (int j = warp; j < rep * HD / 32; j += kAttnThreads / 32) {
            const int kb = kb0 + j;
            encode_block_packed(out[(size_t)b * K + 32 * kb + lane], b, kb, K, planes, lane);
        }
    }
}

// combine splits: out = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s
__global__ void k_attn_merge(const float *__restrict__ part_ml, const float *__restrict__ part_acc, int n_splits,
                             int hd, float *__restrict__ out, int nh, uint8_t *__restrict__ planes) {
    pdl_wait();
    pdl_trigger();
    const int bh = blockIdx.x;   // b * nh + head
    float M = -INFINITY;
    for (int s = 0; s < n_splits; s++) M = fmaxf(M, part_ml[((size_t)bh * n_splits + s) * 2]);
    float L = 0.0f;
    for (int s = 0; s < n_splits; s++) {
        const float m = part_ml[((size_t)bh * n_splits + s) * 2];
        if (m != -INFINITY) L += expf(m - M) * part_ml[((size_t)bh * n_splits + s) * 2 + 1];
    }
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float a = 0.0f;
        for (int s = 0; s < n_splits; s++) {
            const float m = part_ml[((size_t)bh * n_splits + s) * 2];
            if (m != -INFINITY) a += expf(m - M) * part_acc[((size_t)bh * n_splits + s) * hd + d];
        }
        out[(size_t)bh * hd + d] = (L > 0.0f) ? a / L : 0.0f;
    }
    if (planes && hd % 32 == 0) {   // this head's hd / 32 blocks as packed activation rows
        __syncthreads();
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, b = bh / nh, K = nh * hd;
        for (int j = warp; j < hd / 32; j += blockDim.x / 32) {
            const int kb = (bh - b * nh) * hd / 32 + j;
            encode_block_packed(out[(size_t)b * K + 32 * kb + lane], b, kb, K, planes, lane);
        }
    }
}

// KV append: row (b, pos_b) of K and V gets k_new/v_new [B][NKH*HD]
__global__ void k_kv_write(KVView kv, float *k_base, float *v_base, const float *__restrict__ k_new,
                           const float *__restrict__ v_new, const int *__restrict__ pos, int pos_scalar, int row) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const int b = blockIdx.y;
    const int t = pos ? pos[b] : pos_scalar;
    const long long off = kv_offset(kv, b, t);
    if (off < 0) return;
    float *kb = kv.pool_seq ? const_cast<float *>(kv_kbase(kv, b)) : k_base;
    float *vb = kv.pool_seq ? const_cast<float *>(kv_vbase(kv, b)) : v_base;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < row; i += gridDim.x * blockDim.x) {
        kb[off + i] = k_new[(size_t)b * row + i];
        vb[off + i] = v_new[(size_t)b * row + i];
    }
}

static size_t attn_smem(int rep, int hd) {
    return sizeof(float) * ((size_t)rep * hd + kTile * (hd + 1) + kTile * hd + rep * kTile + 3 * rep + 2 * hd);
}

// q [B][nh][hd] -> out [B][nh][hd]; scratch holds the split partials when needed
// programmatic dependent launch (the kernel waits on its predecessor itself, pdl_wait());
// MLQ_NO_PDL=1 launches normally
template <typename... KArgs, typename... Args>
static cudaError_t attn_launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                   Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = getenv("MLQ_NO_PDL") ? 0 : 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

int launch_attn_decode(const float *q, const KVView &kv, const int *seq_lens_dev, int seq_len_scalar,
                       int max_seq_len, int B, int nh, int nkh, int hd, int window, float scale, float *out,
                       float *scratch, size_t scratch_bytes, cudaStream_t s, uint8_t *planes,
                       const AttnRope *rope) {
    if (planes && ((nh / (nkh > 0 ? nkh : 1)) * hd % 32 || hd % 32)) planes = nullptr;   // caller encodes
    AttnRope rp;
    if (rope && rope->pos) {
        if (!kv.pool_seq || rope->rope_dim > hd || rope->rope_dim % 2 || rope->rope_dim <= 0 || !rope->cos_t ||
            !rope->sin_t || !rope->k_new || !rope->v_new)
            return MLQ_ERR_UNSUPPORTED;
        rp = *rope;
    }
    const LaunchEnv *env = launch_env();
    if (!env) return MLQ_ERR_NO_DEVICE;
    if (nkh <= 0 || nh % nkh) { set_error(MLQ_ERR_ARG, "attention: n_head %d not a multiple of n_kv_head %d", nh, nkh); return MLQ_ERR_ARG; }
    const int rep = nh / nkh;
    if ((long long)rep * hd > 16LL * kAttnThreads) {
        set_error(MLQ_ERR_CAPACITY, "attention: n_head/n_kv_head * head_dim = %d > %d", rep * hd, 16 * kAttnThreads);
        return MLQ_ERR_CAPACITY;
    }
    int span = max_seq_len;
    if (window > 0 && span > window) span = window;
    // enough CTAs to cover the SMs: first the positions split, >= 32 (one tile) per split; then,
    // while the CTAs still do not cover the SMs, the query heads of a KV head split over CTAs (each
    // part re-reads the KV tiles, from L2).  Positions first: a tile's fixed cost (its load and
    // three block barriers) is shared by all of a CTA's heads -- heads first made config 3 at
    // 16 sequences 17.5 -> 20.1 ms.  (Config 5's 10 sequences x 2 KV heads had run as 20-40
    // CTAs of 8 query heads each: +120-150 us per attention layer at positions 64-160; config 3
    // at one sequence as 4-8 CTAs.)
    const int ctas = B * nkh;
    int n_splits = 1;
    while (n_splits < 64 && ctas * n_splits < 2 * env->num_sms && span / (n_splits * 2) >= 32) n_splits *= 2;
    int hsplit = 1;
    while (rep % (2 * hsplit) == 0 && ctas * n_splits * hsplit < env->num_sms) hsplit *= 2;
    const int chunk = (span + n_splits - 1) / n_splits;
    const size_t need = (size_t)B * nh * n_splits * (hd + 2) * sizeof(float);
    if (n_splits > 1 && (!scratch || scratch_bytes < need)) n_splits = 1;
    const int chunk1 = n_splits == 1 ? (span > 0 ? span : 1) : chunk;
    float *part_ml = scratch;
    float *part_acc = scratch ? scratch + (size_t)B * nh * n_splits * 2 : nullptr;
    dim3 grid(n_splits, nkh * hsplit, B);
    const size_t smem = attn_smem(rep / hsplit, hd);
#define MLQ_ATTN_CASE(HD_)                                                                                    \
    case HD_: {                                                                                               \
        static bool attr = false;                                                                             \
        if (!attr) {                                                                                          \
            cudaFuncSetAttribute(k_attn_decode<HD_>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024); \
            attr = true;                                                                                      \
        }                                                                                                     \
        if (!MLQ_CUDA(attn_launch_pdl(k_attn_decode<HD_>, grid, dim3(kAttnThreads), smem, s, q, kv,           \
                                      seq_lens_dev, seq_len_scalar, nh, nkh, window, scale, chunk1, out,      \
                                      part_ml, part_acc, planes, rp)))                                        \
            return MLQ_ERR_CUDA;                                                                              \
    } break;
    switch (hd) {
        MLQ_ATTN_CASE(64)
        MLQ_ATTN_CASE(80)
        MLQ_ATTN_CASE(96)
        MLQ_ATTN_CASE(128)
        MLQ_ATTN_CASE(256)
        default:
            set_error(MLQ_ERR_UNSUPPORTED, "attention: head_dim %d (supported 64, 80, 96, 128, 256)", hd);
            return MLQ_ERR_UNSUPPORTED;
    }
#undef MLQ_ATTN_CASE
    count_launch();
    if (n_splits > 1) {
        if (!MLQ_CUDA(attn_launch_pdl(k_attn_merge, dim3(B * nh), dim3(128), 0, s, (const float *)part_ml,
                                      (const float *)part_acc, n_splits, hd, out, nh, planes)))
            return MLQ_ERR_CUDA;
        count_launch();
    }
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

// The decode step's RoPE and KV store in one launch, one CTA per sequence b: q and k rotated
// in place (NeoX halves of the first rope_dim dims of each head, as k_rope_neox, cengine_
// batch_instr.c:686), then the new k / v rows into the cache at position pos[b] (as
// k_kv_write) and, when mirror arrays are given, into the KVBlock's own 64-slot arrays
// ([L][1024][64][row], cengine_batch_instr.c:1349-1350).
__global__ void __launch_bounds__(256) k_rope_kv(float *__restrict__ q, float *__restrict__ k,
                                                 const float *__restrict__ v, int nh, int nkh, int hd, int rope_dim,
                                                 const int *__restrict__ pos, const float *__restrict__ cos_t,
                                                 const float *__restrict__ sin_t, KVView kv,
                                                 float *const *__restrict__ mk, float *const *__restrict__ mv) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x, p = pos[b], hd2 = rope_dim / 2, row = nkh * hd;
    float *qb = q + (size_t)b * nh * hd, *kb = k + (size_t)b * row;
    const float *cs = cos_t + (size_t)p * hd2, *sn = sin_t + (size_t)p * hd2;
    for (int t = threadIdx.x; t < (nh + nkh) * hd2; t += blockDim.x) {
        const int hh = t / hd2, j = t - hh * hd2;
        float *w = hh < nh ? qb + (size_t)hh * hd : kb + (size_t)(hh - nh) * hd;
        const float c = cs[j], sv = sn[j];
        const float a0 = w[j], a1 = w[j + hd2];
        w[j] = a0 * c - a1 * sv;
        w[j + hd2] = a1 * c + a0 * sv;
    }
    __syncthreads();
    const long long off = kv_offset(kv, b, p);
    if (off < 0) return;   // after the block-wide RoPE above; nothing below synchronises
    float *kc = const_cast<float *>(kv_kbase(kv, b)), *vc = const_cast<float *>(kv_vbase(kv, b));
    float *mkb = mk ? mk[b] : nullptr, *mvb = mv ? mv[b] : nullptr;
    size_t moff = 0;
    bool mirror = mkb && mvb && kv.table;
    if (mirror) {
        const int page = kv.table[(size_t)b * kv.table_stride + p / kv.page_size];
        mirror = page >= 0 && page < 1024;
        moff = ((size_t)kv.layer * 1024 * 64 + (size_t)page * 64 + (p % kv.page_size)) * row;
    }
    for (int i = threadIdx.x; i < row; i += blockDim.x) {
        const float kv_k = kb[i], kv_v = v[(size_t)b * row + i];
        kc[off + i] = kv_k;
        vc[off + i] = kv_v;
        if (mirror) {
            mkb[moff + i] = kv_k;
            mvb[moff + i] = kv_v;
        }
    }
}

int launch_rope_kv(float *q, float *k, const float *v, int B, int nh, int nkh, int hd, int rope_dim, const int *pos,
                   const float *cos_t, const float *sin_t, const KVView &kv, float *const *mk, float *const *mv,
                   cudaStream_t s) {
    if (!kv.pool_seq || rope_dim > hd || rope_dim % 2 || !pos) return MLQ_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(B);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = getenv("MLQ_NO_PDL") ? 0 : 1;
    count_launch();
    return MLQ_CUDA(cudaLaunchKernelEx(&cfg, k_rope_kv, q, k, v, nh, nkh, hd, rope_dim, pos, cos_t, sin_t, kv, mk,
                                       mv))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

int launch_kv_write(const KVView &kv, float *k_base, float *v_base, const float *k_new, const float *v_new,
                    const int *pos_dev, int pos_scalar, int B, int row, cudaStream_t s) {
    dim3 grid((row + 255) / 256, B);
    return MLQ_CUDA(launch_pdl_k(k_kv_write, dim3(grid), dim3(256), 0, s, kv, k_base, v_base, k_new, v_new, pos_dev, pos_scalar, row)) ? MLQ_OK : MLQ_ERR_CUDA;
}

size_t attn_scratch_bytes(int B, int nh, int hd) { return (size_t)B * nh * 64 * (hd + 2) * sizeof(float); }

}  // namespace mlq

// ====================================================================================== C-ABI
using namespace mlq;

extern "C" {

// flat KV: k_cache/v_cache [seq_len][n_kv_head * head_dim]
int mlq_attn_decode_flat(const float *q, const float *k_cache, const float *v_cache, float *out, int seq_len,
                         int n_head, int n_kv_head, int head_dim, int window) {
    if (!q || !k_cache || !v_cache || !out || seq_len <= 0 || n_head <= 0 || n_kv_head <= 0 || head_dim <= 0) {
        set_error(MLQ_ERR_ARG, "mlq_attn_decode_flat: bad arguments");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    const size_t kvb = sizeof(float) * (size_t)seq_len * n_kv_head * head_dim;
    const float *dq = (const float *)cs.in(q, sizeof(float) * (size_t)n_head * head_dim);
    const float *dk = (const float *)cs.in(k_cache, kvb);
    const float *dv = (const float *)cs.in(v_cache, kvb);
    float *dout = (float *)cs.out(out, sizeof(float) * (size_t)n_head * head_dim);
    const size_t sb = attn_scratch_bytes(1, n_head, head_dim);
    float *scr = (float *)cs.scratch(sb);
    if (cs.failed) return cs.finish();
    KVView kv{dk, dv, nullptr, 0, 0, 1 << 30, n_kv_head * head_dim, nullptr, 0, 0, 0};
    int rc = launch_attn_decode(dq, kv, nullptr, seq_len, seq_len, 1, n_head, n_kv_head, head_dim, window,
                                1.0f / sqrtf((float)head_dim), dout, scr, sb, stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

// paged KV: pages hold [n_pages][page_size][n_kv_head*head_dim] for K (at k_pages) and V
// (at v_pages); table [B][table_stride] maps logical -> physical pages; seq_lens [B]
int mlq_attn_decode_paged(const float *q, const float *k_pages, const float *v_pages, const int *table,
                          int table_stride, int page_size, int n_pages, const int *seq_lens, int B, int n_head,
                          int n_kv_head, int head_dim, int window, float *out) {
    if (!q || !k_pages || !v_pages || !table || !seq_lens || !out || B <= 0 || page_size <= 0 || n_pages <= 0 ||
        table_stride <= 0 || n_head <= 0 || n_kv_head <= 0 || head_dim <= 0) {
        set_error(MLQ_ERR_ARG, "mlq_attn_decode_paged: bad arguments");
        return MLQ_ERR_ARG;
    }
    int max_len = 0;
    const bool host_lens = !is_device_ptr(seq_lens);
    if (host_lens) {
        for (int b = 0; b < B; b++) {
            if (seq_lens[b] < 0 || seq_lens[b] > table_stride * page_size) {
                set_error(MLQ_ERR_CAPACITY, "mlq_attn_decode_paged: seq_len %d beyond the page table", seq_lens[b]);
                return MLQ_ERR_CAPACITY;
            }
            if (seq_lens[b] > max_len) max_len = seq_lens[b];
        }
    } else {
        max_len = table_stride * page_size;
    }
    // a host table is checked here, before anything is launched: every page a sequence
    // reads (its first ceil(seq_len / page_size) entries; all of them when the lengths
    // are on the device) must name a page of the pool
    if (!is_device_ptr(table)) {
        for (int b = 0; b < B; b++) {
            const int used = host_lens ? (seq_lens[b] + page_size - 1) / page_size : table_stride;
            for (int i = 0; i < used; i++) {
                const int pg = table[(size_t)b * table_stride + i];
                if (pg < 0 || pg >= n_pages) {
                    set_error(MLQ_ERR_ARG, "mlq_attn_decode_paged: sequence %d, logical page %d -> page %d outside "
                              "the pool of %d pages", b, i, pg, n_pages);
                    return MLQ_ERR_ARG;
                }
            }
        }
    }
    CallScope cs;
    const size_t pool = sizeof(float) * (size_t)n_pages * page_size * n_kv_head * head_dim;
    const float *dq = (const float *)cs.in(q, sizeof(float) * (size_t)B * n_head * head_dim);
    const float *dk = (const float *)cs.in(k_pages, pool);
    const float *dv = (const float *)cs.in(v_pages, pool);
    const int *dt = (const int *)cs.in(table, sizeof(int) * (size_t)B * table_stride);
    const int *dl = (const int *)cs.in(seq_lens, sizeof(int) * (size_t)B);
    float *dout = (float *)cs.out(out, sizeof(float) * (size_t)B * n_head * head_dim);
    const size_t sb = attn_scratch_bytes(B, n_head, head_dim);
    float *scr = (float *)cs.scratch(sb);
    if (cs.failed) return cs.finish();
    KVView kv{dk, dv, dt, table_stride, (long long)page_size * n_kv_head * head_dim, page_size,
              n_kv_head * head_dim, nullptr, 0, 0, 0};
    kv.n_pages = n_pages;   // device tables: a corrupt entry reads zeros, never outside the pool
    int rc = launch_attn_decode(dq, kv, dl, 0, max_len, B, n_head, n_kv_head, head_dim, window,
                                1.0f / sqrtf((float)head_dim), dout, scr, sb, stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

}  // extern "C"
