// qwen36_batch_forward (cengine_batch_instr.c:859-1231): the hybrid SSM/attention MoE
// model's decode step for B tokens in one call, as the reference's Python engine drives it
// (turbo_engine_v7_moe.py:1730-1893: B = len(token_ids), kv_lens advanced by the caller).
//
// Per layer, as the reference computes it:
//   xn = RMSNorm(clamp(x)) * attn_norm  (x itself stays the residual, unclamped)
//   SSM layer (layer_types[l] == 1 and ssm_conv1d[l]):
//     x += W_ssm_out . ((W_attn_gate . xn) * ssm_decode_step(xn))
//   attention layer: qkv = W_qkv . xn; Q = qkv[0:NH*HD], K = qkv[NH*HD : +n_kv], V (below);
//     NeoX RoPE at pos = kv_lens[l] on Q and K; every token of the batch writes its K/V to
//     the same slot pos of the flat cache [L][max_ctx][n_kv] (the last token's row stays)
//     and attends over slots 0..pos-1 plus its own row; x += W_attn_out . att
//   xn = RMSNorm(clamp(x)) * ffn_norm
//   MoE (experts and router present): router GEMV, softmax, insertion top-k, renormalised
//     weights; silu(clamp(gate, +-80)) * up per expert; weighted down sum; shared expert
//     scaled by its router score when positive; x += ffn
// then the final RMSNorm and the logits GEMV; ws[0:B*N] holds x (pre-norm) afterwards.
//
// The V section: the reference reads it at NH*HD + N (it assumes K and V sections N wide,
// :1057-1058).  Default: V starts half-way through the non-Q part of the projection
// (NH*HD + (qkv_nr - NH*HD)/2), which is the same place for the reference's layout
// (qkv_nr = NH*HD + 2N) and the standard one (qkv_nr = NH*HD + 2*n_kv).  With
// mlq_set_ref_compat(1) the reference's offset is used and any part of it beyond the
// projection is read from the caller's workspace, where the reference finds it.
//
// KV cache: kv_k / kv_v may be device or host memory.  Host caches get a device mirror
// (kept per host address) that uploads rows the mirror has not seen below kv_lens[l] and
// writes each step's new row back to the host arrays, so both stay the reference's layout.
// Rows below the last position this library wrote are taken as unchanged unless the first
// or last synchronised row no longer matches the host (a new conversation in reused
// memory), which re-uploads the layer.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <map>
#include <mutex>
#include <vector>

#include "../../include/mojollama_b200.h"
#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

// V slice with an optional fallback source for columns past the projection
__global__ void k_copy_cols_ext(float *__restrict__ dst, const float *__restrict__ src, int n, int src_stride,
                                int off, int src_width, const float *__restrict__ ext) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const int b = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int c = off + i;
        dst[(size_t)b * n + i] = c < src_width ? src[(size_t)b * src_stride + c] : (ext ? ext[c - src_width] : 0.0f);
    }
}

// The batch engine's emb_lookup for emb_quant 12 (cengine_batch_instr.c:708-729) in
// reference-compatibility mode: value = d*(sc-32)/8 * (nibble-8) - dm*(m-32)/8 * 6, low
// nibble of byte j/2 for even j -- not the GGUF Q4_K decode (used otherwise).
__global__ void k_emb_q4k_ref(const uint8_t *__restrict__ emb, const int *__restrict__ tokens, float *__restrict__ x,
                              int N, int V) {
    const int b = blockIdx.y;
    int t = tokens[b];
    if (t < 0 || t >= V) t = 0;
    const int bpr = N / 256;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x) {
        const int bi = i / 256, j = i % 256, g = j / 32;
        const uint8_t *bp = emb + ((size_t)t * bpr + bi) * 144;
        const float d = __half2float(__ushort_as_half((unsigned short)(bp[0] | (bp[1] << 8))));
        const float dm = __half2float(__ushort_as_half((unsigned short)(bp[2] | (bp[3] << 8))));
        const uint8_t *q = bp + 4;
        int sc, mn;
        if (g < 4) {
            sc = q[g] & 63;
            mn = q[g + 4] & 63;
        } else {
            sc = (q[g + 4] & 0xF) | ((q[g - 4] >> 6) << 4);
            mn = (q[g + 4] >> 4) | ((q[g] >> 6) << 4);
        }
        const float d_sc = d * (float)(sc - 32) / 8.0f;
        const float d_mn = dm * (float)(mn - 32) / 8.0f;
        const int s = (bp[16 + j / 2] >> ((j & 1) * 4)) & 0xF;
        x[(size_t)b * N + i] = d_sc * (float)(s - 8) - d_mn * 6.0f;
    }
}

__global__ void k_embed_rows(const float *__restrict__ emb, const int *__restrict__ tokens, float *__restrict__ x,
                             int N, int V) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const int b = blockIdx.y;
    int t = tokens[b];
    if (t < 0 || t >= V) t = 0;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x)
        x[(size_t)b * N + i] = emb[(size_t)t * N + i];
}

__global__ void k_shexp_score(const float *__restrict__ xn, const float *__restrict__ r, float *__restrict__ score,
                              int N) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    __shared__ float sh[32];
    const int b = blockIdx.x;
    float s = 0.0f;
    for (int i = threadIdx.x; i < N; i += blockDim.x) s = fmaf(xn[(size_t)b * N + i], r[i], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) score[b] = s;
    }
}

__global__ void k_add_scaled_if_pos(float *__restrict__ x, const float *__restrict__ y, const float *__restrict__ score,
                                    int N) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const int b = blockIdx.y;
    const float sc = score[b];
    if (!(sc > 0.0f)) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x)
        x[(size_t)b * N + i] += sc * y[(size_t)b * N + i];
}

static int grid_cols(long long n) {
    long long g = (n + 255) / 256;
    return (int)(g > 16 ? 16 : (g < 1 ? 1 : g));
}

// Embedding rows of the batch engines (emb_lookup, cengine_batch_instr.c:708-729): a Q4_K
// table when emb_quant is 12 (GGUF decode, or the reference's own formula in
// reference-compatibility mode), fp32 rows for every other value.  emb is the device copy
// of the table; d_tok device token ids, h_tok the same ids on the host.
int launch_embed(const void *emb, int emb_quant, const int *d_tok, const int *h_tok, float *x, int B, int N, int V,
                 cudaStream_t s) {
    if (emb_quant == MLQ_Q4_K) {
        if (N % 256) {
            set_error(MLQ_ERR_ARG, "Q4_K embedding needs N %% 256 == 0 (N = %d)", N);
            return MLQ_ERR_ARG;
        }
        if (ref_compat()) {
            k_emb_q4k_ref<<<dim3(grid_cols(N), B), 256, 0, s>>>((const uint8_t *)emb, d_tok, x, N, V);
            count_launch();
            return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
        }
        const size_t rb = mlq_row_bytes(MLQ_Q4_K, N);
        for (int b = 0; b < B; b++) {
            const int t = (h_tok[b] < 0 || h_tok[b] >= V) ? 0 : h_tok[b];
            const int rc = launch_dequantize((const uint8_t *)emb + rb * (size_t)t, MLQ_Q4_K, x + (size_t)b * N, N, s);
            if (rc != MLQ_OK) return rc;
        }
        return MLQ_OK;
    }
    return MLQ_CUDA(launch_pdl_k(k_embed_rows, dim3(dim3(grid_cols(N), B)), dim3(256), 0, s, (const float *)emb, d_tok, x, N, V)) ? MLQ_OK : MLQ_ERR_CUDA;
}

size_t embed_bytes(int emb_quant, int N, int V) {
    return emb_quant == MLQ_Q4_K ? mlq_row_bytes(MLQ_Q4_K, N) * (size_t)V : sizeof(float) * (size_t)N * V;
}

// token ids on the host, whether the caller passed host or device memory
bool host_tokens(const int *tokens, int B, std::vector<int> &out) {
    out.resize(B);
    if (is_device_ptr(tokens)) return MLQ_CUDA(cudaMemcpy(out.data(), tokens, sizeof(int) * B, cudaMemcpyDeviceToHost));
    memcpy(out.data(), tokens, sizeof(int) * B);
    return true;
}

// ------------------------------------------------------------------------------ KV mirrors
struct KvMirror {
    float *dk = nullptr, *dv = nullptr;
    size_t floats = 0;
    int L = 0, max_ctx = 0, n_kv = 0;
    std::vector<int> wm;                       // rows [0, wm[l]) of layer l are in the mirror
    std::vector<std::vector<float>> first, last;   // host row 0 and row wm-1 (K) when synced
};
static std::mutex g_mirror_mu;
static std::map<std::pair<int, uintptr_t>, KvMirror> g_mirrors;

static void free_mirror(KvMirror &m) {
    if (m.dk) cudaFree(m.dk);
    if (m.dv) cudaFree(m.dv);
    m.dk = m.dv = nullptr;
}

static KvMirror *get_mirror(int dev, const float *hk, int L, int max_ctx, int n_kv) {
    auto key = std::make_pair(dev, (uintptr_t)hk);
    auto it = g_mirrors.find(key);
    if (it != g_mirrors.end() && (it->second.L != L || it->second.max_ctx != max_ctx || it->second.n_kv != n_kv)) {
        free_mirror(it->second);
        g_mirrors.erase(it);
        it = g_mirrors.end();
    }
    if (it == g_mirrors.end()) {
        KvMirror m;
        m.L = L;
        m.max_ctx = max_ctx;
        m.n_kv = n_kv;
        m.floats = (size_t)L * max_ctx * n_kv;
        if (!MLQ_CUDA(cudaMalloc(&m.dk, m.floats * sizeof(float)))) return nullptr;
        if (!MLQ_CUDA(cudaMalloc(&m.dv, m.floats * sizeof(float)))) {
            cudaFree(m.dk);
            return nullptr;
        }
        m.wm.assign(L, 0);
        m.first.assign(L, {});
        m.last.assign(L, {});
        it = g_mirrors.emplace(key, std::move(m)).first;
    }
    return &it->second;
}

void forget_kv_mirrors() {
    std::lock_guard<std::mutex> lk(g_mirror_mu);
    for (auto &kv : g_mirrors) free_mirror(kv.second);
    g_mirrors.clear();
}

// bring layer l's rows [0, pos) of the host cache into the mirror
static bool sync_rows(KvMirror &m, const float *hk, const float *hv, int l, int pos, cudaStream_t s) {
    const size_t row = (size_t)m.n_kv;
    const float *hk_l = hk + (size_t)l * m.max_ctx * row;
    const float *hv_l = hv + (size_t)l * m.max_ctx * row;
    int &wm = m.wm[l];
    if (wm > pos) wm = pos;
    if (wm > 0) {
        const bool same = m.first[l].size() == row && !memcmp(m.first[l].data(), hk_l, row * sizeof(float)) &&
                          m.last[l].size() == row && !memcmp(m.last[l].data(), hk_l + (size_t)(wm - 1) * row,
                                                              row * sizeof(float));
        if (!same) wm = 0;
    }
    if (wm < pos) {
        const size_t off = (size_t)l * m.max_ctx * row + (size_t)wm * row;
        const size_t bytes = (size_t)(pos - wm) * row * sizeof(float);
        if (!MLQ_CUDA(cudaMemcpyAsync(m.dk + off, hk + off, bytes, cudaMemcpyHostToDevice, s))) return false;
        if (!MLQ_CUDA(cudaMemcpyAsync(m.dv + off, hv + off, bytes, cudaMemcpyHostToDevice, s))) return false;
        wm = pos;
    }
    return true;
}

static long long ref_expert_stride(int qt, int rows, int cols) {
    // EXPERT_STRIDE (cengine_batch_instr.c:980-987): unknown types give stride 0
    switch (qt) {
        case MLQ_Q4_K: return (long long)rows * (cols / 256) * 144;
        case MLQ_Q5_K: return (long long)rows * (cols / 256) * 176;
        case MLQ_Q6_K: return (long long)rows * (cols / 256) * 210;
        case MLQ_MXFP4: return (long long)rows * (cols / 32) * 17;
        case MLQ_Q4_0: return (long long)rows * (cols / 32) * 18;
        case MLQ_Q8_0: return (long long)rows * (cols / 32) * 34;
        default: return 0;
    }
}

}  // namespace mlq

using namespace mlq;

extern "C" {

int mlq_qwen36_batch_forward(const MlqQwen36Args *a) {
    if (!a || a->B <= 0 || a->B > 64 || a->L <= 0 || a->N <= 0 || a->N % 32 || a->NH <= 0 || a->n_kv_h <= 0 ||
        a->NH % a->n_kv_h || a->HD <= 0 || !a->tokens || !a->logits || !a->emb || !a->attn_norm_w ||
        !a->ffn_norm_w || !a->out_norm_w || !a->out_w || a->max_ctx <= 0 || !a->cos_table || !a->sin_table) {
        set_error(MLQ_ERR_ARG, "qwen36_batch_forward: bad arguments");
        return MLQ_ERR_ARG;
    }
    const int B = a->B, L = a->L, N = a->N, NH = a->NH, HD = a->HD, nkh = a->n_kv_h;
    const int inner = NH * HD, n_kv = nkh * HD;
    const int rope_dim = a->rope_dim > 0 ? a->rope_dim : HD;
    const bool compat = ref_compat();
    const int si_def = a->shexp_int ? a->shexp_int[0] : 512;
    int S = N;   // workspace slice width (cengine_batch_instr.c:910-918)
    if (inner > S) S = inner;
    if (a->FF > S) S = a->FF;
    if (n_kv > S) S = n_kv;
    if (inner + 2 * n_kv > S) S = inner + 2 * n_kv;
    if (a->n_ff_expert > S) S = a->n_ff_expert;
    if (si_def > S) S = si_def;
    if (S < 8192) S = 8192;
    Ctx *cx = ctx();
    if (!cx) return mlq_last_error();
    CallScope cs;
    cudaStream_t s = stream();

    // ---------------------------------------------------------------- layer checks, sizes
    bool any_attn = false, any_ssm = false;
    int max_qkv = inner, max_gate = 0, max_si = 0, max_nff = a->n_ff_expert > 0 ? a->n_ff_expert : 1;
    for (int l = 0; l < L; l++) {
        const bool ssm = a->layer_types && a->layer_types[l] == 1 && a->ssm_conv1d && a->ssm_conv1d[l];
        if (ssm) {
            any_ssm = true;
            if (!a->attn_gate_raw || !a->attn_gate_raw[l] || !a->ssm_out_raw || !a->ssm_out_raw[l] ||
                a->gate_nc[l] != N || a->gate_nr[l] > a->ssm_inner || a->ssm_out_nc[l] != a->ssm_inner ||
                a->ssm_out_nr[l] != N || !a->ssm_state || a->ssm_inner <= 0) {
                set_error(MLQ_ERR_ARG, "qwen36_batch_forward: SSM layer %d weights or sizes", l);
                return MLQ_ERR_ARG;
            }
            if (a->gate_nr[l] > max_gate) max_gate = a->gate_nr[l];
        } else {
            any_attn = true;
            if (!a->attn_qkv_raw || !a->attn_qkv_raw[l] || !a->attn_out_raw || !a->attn_out_raw[l] ||
                a->qkv_nc[l] != N || a->qkv_nr[l] < inner + 2 * n_kv || a->out_nc[l] != inner || a->out_nr[l] != N) {
                set_error(MLQ_ERR_ARG, "qwen36_batch_forward: attention layer %d weights or sizes", l);
                return MLQ_ERR_ARG;
            }
            if (a->qkv_nr[l] > max_qkv) max_qkv = a->qkv_nr[l];
            if (!a->kv_k || !a->kv_v || !a->kv_lens || a->kv_lens[l] < 0 || a->kv_lens[l] >= a->max_ctx) {
                set_error(MLQ_ERR_CAPACITY, "qwen36_batch_forward: layer %d position %d (max_ctx %d)", l,
                          a->kv_lens ? a->kv_lens[l] : -1, a->max_ctx);
                return MLQ_ERR_CAPACITY;
            }
        }
        if (a->shexp_router && a->shexp_router[l]) {
            const int si = a->shexp_int ? a->shexp_int[l] : 512;
            if (si > max_si) max_si = si;
        }
    }
    const int E = a->n_experts, topk = a->top_k, M = a->n_ff_expert;
    if (E > 0 && topk > 0 && (topk > 16 || topk > E || M <= 0)) {
        set_error(MLQ_ERR_ARG, "qwen36_batch_forward: top_k %d of %d experts", topk, E);
        return MLQ_ERR_ARG;
    }

    // ---------------------------------------------------------------- buffers
    const int wide = max_qkv > inner + N + n_kv ? max_qkv : inner + N + n_kv;
    int *d_tok = (int *)cs.in(a->tokens, sizeof(int) * B);
    float *x = (float *)cs.scratch(sizeof(float) * (size_t)B * N);
    float *xn = (float *)cs.scratch(sizeof(float) * (size_t)B * N);
    float *qkv = (float *)cs.scratch(sizeof(float) * (size_t)B * max_qkv);
    float *q = (float *)cs.scratch(sizeof(float) * (size_t)B * inner);
    float *k = (float *)cs.scratch(sizeof(float) * (size_t)B * n_kv);
    float *v = (float *)cs.scratch(sizeof(float) * (size_t)B * n_kv);
    const int wbuf = inner > a->ssm_inner ? inner : a->ssm_inner;
    float *att = (float *)cs.scratch(sizeof(float) * (size_t)B * (wbuf > 0 ? wbuf : 1));
    float *g = (float *)cs.scratch(sizeof(float) * (size_t)B * (wbuf > max_si ? wbuf : max_si));
    float *u = (float *)cs.scratch(sizeof(float) * (size_t)B * (max_si > 0 ? max_si : 1));
    float *tmp = (float *)cs.scratch(sizeof(float) * (size_t)B * N);
    float *lg = (float *)cs.scratch(sizeof(float) * (size_t)B * (E > 0 ? E : 1));
    int *e_idx = (int *)cs.scratch(sizeof(int) * (size_t)B * (topk > 0 ? topk : 1));
    float *e_w = (float *)cs.scratch(sizeof(float) * (size_t)B * (topk > 0 ? topk : 1));
    float *hm = (float *)cs.scratch(sizeof(float) * (size_t)B * (topk > 0 ? topk : 1) * max_nff);
    float *hm2 = (float *)cs.scratch(sizeof(float) * (size_t)B * (topk > 0 ? topk : 1) * max_nff);
    float *score = (float *)cs.scratch(sizeof(float) * B);
    const size_t attn_sb = attn_scratch_bytes(B, NH, HD);
    float *attn_scr = (float *)cs.scratch(attn_sb);
    // shared experts on the block-scaled tensor cores: the rows' E2M1 planes (input, SwiGLU)
    uint8_t *shp_x = nullptr, *shp_h = nullptr;
    if (max_si > 0 && B >= 2) {
        shp_x = (uint8_t *)cs.scratch(mxf4_planes_bytes(B, N));
        shp_h = (uint8_t *)cs.scratch(mxf4_planes_bytes(B, max_si));
    }
    // reference-compatibility V columns beyond the projection come from ws's qkv slice
    const float *v_ext = nullptr;
    if (compat && any_attn && a->ws) {
        int minq = max_qkv;
        for (int l = 0; l < L; l++)
            if (!(a->layer_types && a->layer_types[l] == 1) && a->qkv_nr[l] < minq) minq = a->qkv_nr[l];
        if (inner + N + n_kv > minq)
            v_ext = (const float *)cs.in(a->ws + (size_t)3 * B * S, sizeof(float) * (size_t)wide);
    }
    float *d_state = any_ssm ? (float *)cs.inout(a->ssm_state, sizeof(float) * (size_t)L * a->ssm_groups *
                                                                    a->ssm_state_size)
                             : nullptr;
    float *d_logits = (float *)cs.out(a->logits, sizeof(float) * (size_t)B * a->out_nr_final);
    float *ws_out = a->ws ? (float *)cs.out(a->ws, sizeof(float) * (size_t)B * N) : nullptr;
    if (cs.failed) return cs.finish();

    // KV cache: device arrays directly, host arrays through the mirror
    float *dk = a->kv_k, *dv = a->kv_v;
    KvMirror *mir = nullptr;
    std::unique_lock<std::mutex> mlk(g_mirror_mu, std::defer_lock);
    if (any_attn && !(is_device_ptr(a->kv_k) && is_device_ptr(a->kv_v))) {
        mlk.lock();
        mir = get_mirror(cx->device, a->kv_k, L, a->max_ctx, n_kv);
        if (!mir) {
            cs.failed = true;
            cs.finish();
            return mlq_last_error();
        }
        dk = mir->dk;
        dv = mir->dv;
        for (int l = 0; l < L; l++) {
            if (a->layer_types && a->layer_types[l] == 1 && a->ssm_conv1d && a->ssm_conv1d[l]) continue;
            if (!sync_rows(*mir, a->kv_k, a->kv_v, l, a->kv_lens[l], s)) {
                cs.failed = true;
                cs.finish();
                return MLQ_ERR_CUDA;
            }
        }
    }

    int rc = MLQ_OK;
#define MLQ_TRY(expr)                  \
    do {                               \
        if (rc == MLQ_OK) rc = (expr); \
    } while (0)
    // ---------------------------------------------------------------- embedding
    {
        // the vocabulary is the output projection's row count (the reference reads emb[token])
        const int V = a->out_nr_final;
        std::vector<int> th(B, 0);   // host ids are needed only by the per-row Q4_K decode
        const void *emb = cs.weights(a->emb, embed_bytes(a->emb_quant, N, V));
        if (!emb || (a->emb_quant == MLQ_Q4_K && !compat && !host_tokens(a->tokens, B, th)))
            rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG;
        MLQ_TRY(launch_embed(emb, a->emb_quant, d_tok, th.data(), x, B, N, V, s));
    }
    const float scale = 1.0f / sqrtf((float)HD);
    const float *cos_t = (const float *)cs.weights(a->cos_table, sizeof(float) * (size_t)a->max_ctx * (rope_dim / 2));
    const float *sin_t = (const float *)cs.weights(a->sin_table, sizeof(float) * (size_t)a->max_ctx * (rope_dim / 2));
    if (cs.failed && rc == MLQ_OK) rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG;

    // ---------------------------------------------------------------- layers
    for (int l = 0; l < L && rc == MLQ_OK; l++) {
        const bool ssm = a->layer_types && a->layer_types[l] == 1 && a->ssm_conv1d && a->ssm_conv1d[l];
        const float *an = (const float *)cs.weights(a->attn_norm_w[l], sizeof(float) * N);
        MLQ_TRY(launch_rms_norm(xn, x, an, nullptr, B, N, a->eps, 1, s));
        if (ssm) {
            const int G = a->ssm_groups, SS = a->ssm_state_size, R = a->ssm_dt_rank, IN = a->ssm_inner;
            const float *conv = (const float *)cs.weights(a->ssm_conv1d[l], sizeof(float) * 2 * (size_t)IN);
            const float *sa = (const float *)cs.weights(a->ssm_a[l], sizeof(float) * G);
            const float *sdt = (const float *)cs.weights(a->ssm_dt_bias[l], sizeof(float) * G);
            const float *sal = (const float *)cs.weights(a->ssm_alpha[l], sizeof(float) * (size_t)G * R);
            const float *sbe = (const float *)cs.weights(a->ssm_beta[l], sizeof(float) * (size_t)G * R);
            const uint8_t *wg = (const uint8_t *)cs.weights(a->attn_gate_raw[l],
                                                            mlq_row_bytes(a->gate_qt[l], N) * (size_t)a->gate_nr[l]);
            const uint8_t *wo = (const uint8_t *)cs.weights(a->ssm_out_raw[l],
                                                            mlq_row_bytes(a->ssm_out_qt[l], IN) * (size_t)N);
            if (cs.failed) { rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG; break; }
            MLQ_TRY(launch_ssm_decode_step(xn, att, conv, sa, sdt, sal, sbe, d_state + (size_t)l * G * SS, B, N, IN, G,
                                           SS, R, s));
            // gate rows land at b*ssm_inner (the reference's stride); rows past gate_nr keep 0
            if (a->gate_nr[l] == IN) {
                MLQ_TRY(launch_matmul(wg, a->gate_qt[l], xn, g, IN, N, B, 0, s));
            } else {
                cudaMemsetAsync(g, 0, sizeof(float) * (size_t)B * IN, s);
                for (int b = 0; b < B; b++)
                    MLQ_TRY(launch_matmul(wg, a->gate_qt[l], xn + (size_t)b * N, g + (size_t)b * IN, a->gate_nr[l], N,
                                          1, 0, s));
            }
            MLQ_TRY(launch_mul(att, g, (long long)B * IN, s));
            MLQ_TRY(launch_matmul(wo, a->ssm_out_qt[l], att, tmp, N, IN, B, 0, s));
        } else {
            const int nq = a->qkv_nr[l];
            const uint8_t *wqkv = (const uint8_t *)cs.weights(a->attn_qkv_raw[l],
                                                              mlq_row_bytes(a->qkv_qt[l], N) * (size_t)nq);
            const uint8_t *wo = (const uint8_t *)cs.weights(a->attn_out_raw[l],
                                                            mlq_row_bytes(a->out_qt[l], inner) * (size_t)N);
            if (cs.failed) { rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG; break; }
            const int pos = a->kv_lens[l];
            MLQ_TRY(launch_matmul(wqkv, a->qkv_qt[l], xn, qkv, nq, N, B, 0, s));
            const int voff = compat ? inner + N : inner + (nq - inner) / 2;
            if (rc == MLQ_OK) {
                const float *none = nullptr, *vx = v_ext ? v_ext + nq : nullptr;
                MLQ_TRY(MLQ_CUDA(launch_pdl_k(k_copy_cols_ext, dim3(grid_cols(inner), B), dim3(256), 0, s, q, qkv, inner,
                                              nq, 0, nq, none)) ? MLQ_OK : MLQ_ERR_CUDA);
                MLQ_TRY(MLQ_CUDA(launch_pdl_k(k_copy_cols_ext, dim3(grid_cols(n_kv), B), dim3(256), 0, s, k, qkv, n_kv,
                                              nq, inner, nq, none)) ? MLQ_OK : MLQ_ERR_CUDA);
                MLQ_TRY(MLQ_CUDA(launch_pdl_k(k_copy_cols_ext, dim3(grid_cols(n_kv), B), dim3(256), 0, s, v, qkv, n_kv,
                                              nq, voff, nq, vx)) ? MLQ_OK : MLQ_ERR_CUDA);
            }
            MLQ_TRY(launch_rope_neox(q, B, inner, NH, HD, nullptr, pos, cos_t, sin_t, rope_dim, s));
            MLQ_TRY(launch_rope_neox(k, B, n_kv, nkh, HD, nullptr, pos, cos_t, sin_t, rope_dim, s));
            float *kl = dk + (size_t)l * a->max_ctx * n_kv, *vl = dv + (size_t)l * a->max_ctx * n_kv;
            // attention: slots 0..pos-1 from the cache, slot pos from each token's own row
            KVView kvv{kl, vl, nullptr, 0, 0, 0, n_kv, nullptr, 0, 0, 0, k, v, n_kv};
            MLQ_TRY(launch_attn_decode(q, kvv, nullptr, pos + 1, pos + 1, B, NH, nkh, HD, 0, scale, att, attn_scr,
                                       attn_sb, s));
            // the cache keeps the last token's row at slot pos, as the reference leaves it
            KVView flat{kl, vl, nullptr, 0, 0, 0, n_kv, nullptr, 0, 0, 0};
            MLQ_TRY(launch_kv_write(flat, kl, vl, k + (size_t)(B - 1) * n_kv, v + (size_t)(B - 1) * n_kv, nullptr, pos,
                                    1, n_kv, s));
            if (mir && rc == MLQ_OK) {
                const size_t off = ((size_t)l * a->max_ctx + pos) * n_kv;
                if (!MLQ_CUDA(cudaMemcpyAsync(a->kv_k + off, dk + off, n_kv * sizeof(float), cudaMemcpyDeviceToHost, s)) ||
                    !MLQ_CUDA(cudaMemcpyAsync(a->kv_v + off, dv + off, n_kv * sizeof(float), cudaMemcpyDeviceToHost, s)))
                    rc = MLQ_ERR_CUDA;
            }
            MLQ_TRY(launch_matmul(wo, a->out_qt[l], att, tmp, N, inner, B, 0, s));
        }
        // FFN
        const float *fnw = (const float *)cs.weights(a->ffn_norm_w[l], sizeof(float) * N);
        // x += the block's output (tmp), then the FFN norm, in one launch
        MLQ_TRY(launch_add_rms_norm(x, tmp, fnw, xn, B, N, a->eps, 1, s));
        const bool has_moe = E > 0 && topk > 0 && a->gate_exp_raw && a->gate_exp_raw[l] && a->moe_router_raw &&
                             a->moe_router_raw[l];
        if (!has_moe || rc != MLQ_OK) continue;
        const int gqt = a->gate_exp_qt ? a->gate_exp_qt[l] : MLQ_Q4_K;
        const int uqt = a->up_exp_qt ? a->up_exp_qt[l] : MLQ_Q4_K;
        const int dqt = a->down_exp_qt ? a->down_exp_qt[l] : MLQ_Q6_K;
        const int rqt = a->moe_router_qt ? a->moe_router_qt[l] : MLQ_F32;
        const long long gs = compat ? ref_expert_stride(gqt, M, N) : (long long)M * mlq_row_bytes(gqt, N);
        const long long us = compat ? ref_expert_stride(uqt, M, N) : (long long)M * mlq_row_bytes(uqt, N);
        const long long ds = compat ? ref_expert_stride(dqt, N, M) : (long long)N * mlq_row_bytes(dqt, M);
        const size_t gm = (size_t)M * mlq_row_bytes(gqt, N), um = (size_t)M * mlq_row_bytes(uqt, N),
                     dm = (size_t)N * mlq_row_bytes(dqt, M);
        if (!gm || !um || !dm || !mlq_row_bytes(rqt, N)) {
            set_error(MLQ_ERR_TYPE, "qwen36_batch_forward: layer %d expert/router types %d/%d/%d/%d", l, gqt, uqt, dqt,
                      rqt);
            rc = MLQ_ERR_TYPE;
            break;
        }
        auto extent = [&](long long st, size_t mat) { return (size_t)st * (E - 1) + mat; };
        const uint8_t *wr = (const uint8_t *)cs.weights(a->moe_router_raw[l], mlq_row_bytes(rqt, N) * (size_t)E);
        const uint8_t *ge = (const uint8_t *)cs.weights(a->gate_exp_raw[l], extent(gs, gm));
        const uint8_t *ue = (const uint8_t *)cs.weights(a->up_exp_raw[l], extent(us, um));
        const uint8_t *de = (const uint8_t *)cs.weights(a->down_exp_raw[l], extent(ds, dm));
        if (cs.failed) { rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG; break; }
        // an fp32 router and a shared expert: its gate score rides in the router's launch as
        // one more row (the score is used after the routed experts; xn is unchanged until then)
        bool score_done = false;
        if (rqt == MLQ_F32 && a->shexp_router && a->shexp_router[l]) {
            const float *sr = (const float *)cs.weights(a->shexp_router[l], sizeof(float) * N);
            if (cs.failed) { rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG; break; }
            MLQ_TRY(launch_router_rows_f32((const float *)wr, sr, xn, lg, score, E, N, B, s));
            score_done = true;
        } else {
            MLQ_TRY(launch_matmul(wr, rqt, xn, lg, E, N, B, 0, s));
        }
        MLQ_TRY(launch_router_topk(lg, B, E, topk, 1, e_idx, e_w, s));
        const bool grouped = N % 32 == 0 && M % 32 == 0 && E <= 1024 && grouped_tiles_per_expert(gqt, M, N) &&
                             grouped_tiles_per_expert(uqt, M, N) && grouped_tiles_per_expert(dqt, N, M) &&
                             !getenv("MLQ_NO_GROUPED_MOE");
        const bool shexp = a->shexp_router && a->shexp_router[l];
        float *ym = nullptr;   // grouped: the routed rows, combined after the shared expert
        if (grouped && rc == MLQ_OK) {
            // every active expert streamed once for all of its (token, slot) rows, then
            // x += sum_i w_i y_i in slot order (moe_forward_omp's +-80 SiLU clamp)
            const int R = B * topk;
            uint8_t *mscr = (uint8_t *)cs.scratch(moe_grouped_scratch_bytes(gqt, uqt, dqt, R, E, M, N));
            ym = (float *)cs.scratch(sizeof(float) * (size_t)R * N);
            if (cs.failed) { rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_CUDA; break; }
            MoeGroupedScratch ms;
            moe_grouped_carve(ms, mscr, gqt, uqt, dqt, R, E, M, N);
            MLQ_TRY(launch_moe_grouped(gqt, uqt, dqt, ge, ue, de, gs, us, ds, E, e_idx, R, topk, M, N, xn, ym, 80.0f,
                                       ms, s));
            // with a shared expert the combine also adds its scaled output (below): one launch
            if (!shexp) MLQ_TRY(launch_ep_combine(ym, nullptr, e_w, B, topk, N, x, x, s));
        } else {
            MLQ_TRY(launch_moe_experts(gqt, uqt, dqt, ge, ue, de, gs, us, ds, e_idx, e_w, topk, B, M, N, xn, hm, hm2, x,
                                       x, 80.0f, s));
        }
        if (shexp) {
            const int si = a->shexp_int ? a->shexp_int[l] : 512;
            const int sgq = a->shexp_gate_qt ? a->shexp_gate_qt[l] : MLQ_MXFP4;
            const int suq = a->shexp_up_qt ? a->shexp_up_qt[l] : MLQ_MXFP4;
            const int sdq = a->shexp_down_qt ? a->shexp_down_qt[l] : MLQ_MXFP4;
            const float *sr = (const float *)cs.weights(a->shexp_router[l], sizeof(float) * N);
            const uint8_t *sg = (const uint8_t *)cs.weights(a->shexp_gate_raw[l], mlq_row_bytes(sgq, N) * (size_t)si);
            const uint8_t *su = (const uint8_t *)cs.weights(a->shexp_up_raw[l], mlq_row_bytes(suq, N) * (size_t)si);
            const uint8_t *sd = (const uint8_t *)cs.weights(a->shexp_down_raw[l], mlq_row_bytes(sdq, si) * (size_t)N);
            if (cs.failed) { rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG; break; }
            if (!score_done)
                MLQ_TRY(MLQ_CUDA(launch_pdl_k(k_shexp_score, dim3(B), dim3(256), 0, s, xn, sr, score, N)) ? MLQ_OK
                                                                                                            : MLQ_ERR_CUDA);
            if (shp_x && sgq == MLQ_MXFP4 && suq == MLQ_MXFP4 && sdq == MLQ_MXFP4 && si % 32 == 0 &&
                mxf4_dense_supported(sg, si, N) && mxf4_dense_supported(su, si, N) && mxf4_dense_supported(sd, N, si)) {
                // MXFP4 (the GGUF shared-expert type): gate and up in one launch of the grouped
                // block-scaled kernel over all B rows, silu(clamp(g, +-80)) * u encoded, then down
                MLQ_TRY(launch_mxf4_planes_rows(xn, nullptr, nullptr, 1, N, 0.0f, B, N, shp_x, s));
                MLQ_TRY(launch_mxf4_dense_tc(sg, su, si, N, shp_x, B, g, u, s));
                MLQ_TRY(launch_mxf4_planes_rows(g, u, nullptr, 1, si, 80.0f, B, si, shp_h, s));
                MLQ_TRY(launch_mxf4_dense_tc(sd, nullptr, N, si, shp_h, B, tmp, nullptr, s));
            } else {
                MLQ_TRY(launch_matmul(sg, sgq, xn, g, si, N, B, 0, s));
                MLQ_TRY(launch_matmul(su, suq, xn, u, si, N, B, 0, s));
                MLQ_TRY(launch_swiglu(g, g, u, (long long)B * si, s));
                MLQ_TRY(launch_matmul(sd, sdq, g, tmp, N, si, B, 0, s));
            }
            if (ym) {
                // x += sum_i w_i y_i, then x += score * shared where score > 0, in one launch
                MLQ_TRY(launch_ep_combine(ym, nullptr, e_w, B, topk, N, x, x, s, tmp, score));
            } else if (rc == MLQ_OK) {
                MLQ_TRY(MLQ_CUDA(launch_pdl_k(k_add_scaled_if_pos, dim3(grid_cols(N), B), dim3(256), 0, s, x, tmp,
                                              score, N)) ? MLQ_OK : MLQ_ERR_CUDA);
            }
        }
    }
    // ---------------------------------------------------------------- head
    if (rc == MLQ_OK && ws_out) cudaMemcpyAsync(ws_out, x, sizeof(float) * (size_t)B * N, cudaMemcpyDeviceToDevice, s);
    const float *onw = (const float *)cs.weights(a->out_norm_w, sizeof(float) * N);
    const uint8_t *wout = (const uint8_t *)cs.weights(
        a->out_w, mlq_row_bytes(a->out_qt_final, a->out_nc_final) * (size_t)a->out_nr_final);
    if (cs.failed && rc == MLQ_OK) rc = mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG;
    MLQ_TRY(launch_rms_norm(xn, x, onw, nullptr, B, N, a->eps, 1, s));
    MLQ_TRY(launch_matmul(wout, a->out_qt_final, xn, d_logits, a->out_nr_final, a->out_nc_final, B, 0, s));
#undef MLQ_TRY
    if (mir) {
        // rows up to pos of every attention layer are now in the mirror (and on the host)
        for (int l = 0; l < L; l++) {
            if (a->layer_types && a->layer_types[l] == 1 && a->ssm_conv1d && a->ssm_conv1d[l]) continue;
            const int pos = a->kv_lens[l];
            mir->wm[l] = rc == MLQ_OK ? pos + 1 : (mir->wm[l] < pos ? mir->wm[l] : pos);
        }
    }
    if (rc != MLQ_OK) {
        cs.failed = true;
        cs.finish();
        return rc;
    }
    rc = cs.finish();
    if (mir && rc == MLQ_OK) {
        // remember row 0 and the last row of each layer as the host holds them now
        const size_t row = (size_t)n_kv;
        for (int l = 0; l < L; l++) {
            if (a->layer_types && a->layer_types[l] == 1 && a->ssm_conv1d && a->ssm_conv1d[l]) continue;
            const float *hk_l = a->kv_k + (size_t)l * a->max_ctx * row;
            mir->first[l].assign(hk_l, hk_l + row);
            mir->last[l].assign(hk_l + (size_t)(mir->wm[l] - 1) * row, hk_l + (size_t)mir->wm[l] * row);
        }
    }
    return rc;
}

}  // extern "C"
