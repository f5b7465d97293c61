// Whole-model decode step: batch_forward(const BC*, tokens, B, ws)
// (cengine_batch_instr.c:1233-1493) -- B sequences, one new token each.
//
// Per layer, as the reference structures it, but with the normalised activations
// actually feeding the projections (the reference writes its pre-norm output back
// into x and projects an untouched buffer, so every layer adds nothing):
//   xn, res = RMSNorm(clamp(x)) * w_attn_norm, clamp(x)          (NaN -> 0, +-1000)
//   SSM layer (layer_types[l] == 1): x = res + W_ssm_out . ((W_attn_gate . xn) * ssm_step(xn))
//   attention layer: q, k, v from fused QKV / fused QK + V / separate projections;
//     NeoX RoPE at the sequence position; K, V appended to the sequence's KVBlock page
//     pool (page allocated on first touch from its LIFO free list); split-K attention
//     over the pages; x = res + (W_attn_gate or W_o) . att
//   xn, res = RMSNorm(clamp(x)) * w_ffn_norm, clamp(x)
//   MoE (n_experts > 0): F32 router, softmax, top-k without renormalisation (moe_ffn,
//     :615-646), experts through the grouped GEMV with device-side indices, shared expert
//     scaled by its router score when positive (:1440-1452); dense: SiLU(gate)*up, down
//   x = res + ffn
// then seq_len += 1 for every sequence, final RMSNorm and the output projection into
// c->logits [B][outNR].
//
// All weight pointers reachable from the BC (host or device) are resolved once per BC
// into a device plan (host weights uploaded through the residency cache); later calls
// with the same BC contents reuse it.  Weights are treated as immutable while a plan
// exists; mlq_cache_clear() drops the plans with the cache.
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "../../include/mojollama_b200_ref_abi.h"
#include "mlq_internal.h"

namespace mlq {

// ------------------------------------------------------------------------------ kernels
// dst[b][0:n] = src[b*src_stride + off : +n]
__global__ void k_copy_cols(float *__restrict__ dst, const float *__restrict__ src, int n, int src_stride, int off) {
    const int b = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        dst[(size_t)b * n + i] = src[(size_t)b * src_stride + off + i];
}

// h = silu(g) * u, exact, no clamp (cengine_batch_instr.c:1465)
__global__ void k_silu_mul(float *__restrict__ h, const float *__restrict__ g, const float *__restrict__ u, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float gv = g[i];
        h[i] = (gv / (1.0f + expf(-gv))) * u[i];
    }
}

// score[b] = xn[b] . r  (one block per token)
__global__ void k_dot_rows(const float *__restrict__ xn, const float *__restrict__ r, float *__restrict__ score, int N) {
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

// The KVBlock's own k/v arrays ([L][1024][64][row], cengine_batch_instr.c:1349-1350) get the
// same rows as the page pool; pages index them with the fixed 64-slot block size.
__global__ void k_kv_mirror(float *const *__restrict__ mk, float *const *__restrict__ mv,
                            const int *__restrict__ tab, int tab_stride, const int *__restrict__ pos,
                            const float *__restrict__ k, const float *__restrict__ v, int row, int page_size,
                            int layer) {
    const int b = blockIdx.y;
    float *kb = mk[b], *vb = mv[b];
    if (!kb || !vb) return;
    const int p = pos[b];
    const int page = tab[(size_t)b * tab_stride + p / page_size];
    if (page < 0 || page >= 1024) return;
    const size_t off = ((size_t)layer * 1024 * 64 + (size_t)page * 64 + (p % page_size)) * row;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < row; i += gridDim.x * blockDim.x) {
        kb[off + i] = k[(size_t)b * row + i];
        vb[off + i] = v[(size_t)b * row + i];
    }
}

// shared expert input (reference :1446-1447): h = silu(up) * gate
__global__ void k_shexp_act(float *__restrict__ h, const float *__restrict__ gate, const float *__restrict__ up, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float u = up[i];
        h[i] = (u / (1.0f + expf(-u))) * gate[i];
    }
}

// x[b] += score[b] * y[b] when score[b] > 0
__global__ void k_add_scaled_pos(float *__restrict__ x, const float *__restrict__ y, const float *__restrict__ score, int N) {
    const int b = blockIdx.y;
    const float sc = score[b];
    if (!(sc > 0.0f)) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < N; i += gridDim.x * blockDim.x)
        x[(size_t)b * N + i] += sc * y[(size_t)b * N + i];
}

static int grid1(long long n) {
    long long g = (n + 255) / 256;
    return (int)(g > 2048 ? 2048 : (g < 1 ? 1 : g));
}

// ------------------------------------------------------------------------------ plan
struct LayerPlan {
    bool ssm = false;
    const float *an = nullptr, *fn = nullptr;
    const uint8_t *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *wqk = nullptr, *wqkv = nullptr,
                  *wattng = nullptr;
    int qq = 0, qk = 0, qv = 0, qo = 0, qqk = 0, qqkv = 0, qattng = 0;
    int nq = 0, nk = 0, nv = 0, no = 0;
    const uint8_t *wg = nullptr, *wu = nullptr, *wd = nullptr;
    int qg = 0, qu = 0, qd = 0, ng = 0, nu = 0, nd = 0;
    const float *router = nullptr;
    const uint8_t *gexp = nullptr, *uexp = nullptr, *dexp = nullptr;
    long long gstride = 0, ustride = 0, dstride = 0;
    const uint8_t *shg = nullptr, *shu = nullptr, *shd = nullptr;
    int qshg = 0, qshu = 0, qshd = 0;
    const float *shrouter = nullptr;
    const float *conv = nullptr, *ssm_a = nullptr, *ssm_dt = nullptr, *ssm_alpha = nullptr, *ssm_beta = nullptr;
    const uint8_t *wssmout = nullptr;
    int qssmout = 0;
    int window = 0;   // attention over the last `window` positions only (0: all)
};

// Per-layer sliding windows of a model description (mlq_set_attention_windows), keyed by
// the BC's address; part of the plan's fingerprint, so changing them rebuilds the plan
static std::mutex g_win_mu;
static std::map<uintptr_t, std::vector<int>> g_windows;

static std::vector<int> windows_of(const BC *c) {
    std::lock_guard<std::mutex> lk(g_win_mu);
    auto it = g_windows.find((uintptr_t)c);
    return it == g_windows.end() ? std::vector<int>() : it->second;
}

struct ModelPlan {
    unsigned long long gen = 0;   // distinguishes rebuilt plans of one BC address
    std::vector<uint8_t> fingerprint;
    std::vector<LayerPlan> layers;
    const float *emb = nullptr;
    const float *onw = nullptr;
    const uint8_t *wout = nullptr;
    const float *cos_t = nullptr, *sin_t = nullptr;
    float *ssm_state = nullptr;   // device view of c->ssm_state (host state is staged per call)
};

static std::mutex g_plan_mu;
static std::map<std::pair<int, uintptr_t>, ModelPlan> g_plans;

// SSM dims hard-coded by the reference engine (cengine_batch_instr.c:1253-1254)
constexpr int kSsmGroups = 32, kSsmState = 128, kSsmDtRank = 32;
constexpr int kShexpFF = 512;   // shared expert width (cengine_batch_instr.c:1444)

template <typename T>
static void fp_push(std::vector<uint8_t> &f, const T *arr, int n) {
    const uint8_t *p = reinterpret_cast<const uint8_t *>(&arr);
    f.insert(f.end(), p, p + sizeof(arr));
    if (arr) {
        const uint8_t *q = reinterpret_cast<const uint8_t *>(arr);
        f.insert(f.end(), q, q + sizeof(T) * (size_t)n);
    }
}

// The per-call members (KV blocks, logits, workspace, SSM state) are left out, so a caller
// that swaps them between steps keeps its plan.
static std::vector<uint8_t> fingerprint(const BC *c) {
    BC k = *c;
    k.kv_array = nullptr;
    k.logits = nullptr;
    k.workspace = nullptr;
    k.ws_size = 0;
    k.ssm_state = nullptr;
    std::vector<uint8_t> f(reinterpret_cast<const uint8_t *>(&k), reinterpret_cast<const uint8_t *>(&k) + sizeof(BC));
    const int L = c->L;
    f.push_back(ref_compat() ? 1 : 0);
    for (int w : windows_of(c)) {
        const uint8_t *wb = reinterpret_cast<const uint8_t *>(&w);
        f.insert(f.end(), wb, wb + sizeof(int));
    }
    fp_push(f, c->wQ, L); fp_push(f, c->wK, L); fp_push(f, c->wV, L); fp_push(f, c->wO, L);
    fp_push(f, c->wG, L); fp_push(f, c->wU, L); fp_push(f, c->wD, L); fp_push(f, c->wAN, L); fp_push(f, c->wFN, L);
    fp_push(f, c->q_quant, L); fp_push(f, c->k_quant, L); fp_push(f, c->v_quant, L); fp_push(f, c->o_quant, L);
    fp_push(f, c->g_quant, L); fp_push(f, c->u_quant, L); fp_push(f, c->d_quant, L);
    fp_push(f, c->nQ, L); fp_push(f, c->nK, L); fp_push(f, c->nV, L); fp_push(f, c->nO, L);
    fp_push(f, c->nG, L); fp_push(f, c->nU, L); fp_push(f, c->nD, L);
    fp_push(f, c->w_gate_inp, L); fp_push(f, c->w_gate_exps, L); fp_push(f, c->w_up_exps, L);
    fp_push(f, c->w_down_exps, L); fp_push(f, c->wQK, L); fp_push(f, c->qk_quant, L); fp_push(f, c->wQKV, L);
    fp_push(f, c->qkv_quant, L); fp_push(f, c->wAttnG, L); fp_push(f, c->attnG_quant, L);
    fp_push(f, c->ssm_conv1d, L); fp_push(f, c->wSsmOut, L); fp_push(f, c->layer_types, L);
    fp_push(f, c->wSHexpG, L); fp_push(f, c->wShexpRouter, L);
    return f;
}

static const uint8_t *W(CallScope &cs, const void *p, int qt, int rows, int cols) {
    if (!p) return nullptr;
    const size_t rb = mlq_row_bytes(qt, cols);
    if (!rb || rows <= 0) {
        set_error(MLQ_ERR_TYPE, "batch_forward: weight type %d with %d x %d", qt, rows, cols);
        cs.failed = true;
        return nullptr;
    }
    return (const uint8_t *)cs.weights(p, rb * (size_t)rows);
}

static const float *Fv(CallScope &cs, const void *p, size_t n) {
    return p ? (const float *)cs.weights(p, sizeof(float) * n) : nullptr;
}

static int at(const int *a, int l, int dflt) { return a ? a[l] : dflt; }

// Bytes between experts of a 3-D expert tensor [E][rows][cols].  Default: the type's row
// size.  Reference-compatibility mode: moe_ffn's own rule (cengine_batch_instr.c:592-604),
// which knows Q4_K/Q5_K/Q6_K/MXFP4 only and uses the Q4_K size for any other gate/up type
// and the Q6_K size for any other down type (integer division by the 256-wide super-block).
static long long expert_stride(int qt, int rows, int cols, bool down) {
    if (!ref_compat()) return (long long)rows * mlq_row_bytes(qt, cols);
    if (qt == MLQ_MXFP4) return (long long)rows * (cols / 32) * 17;
    int bytes = down ? 210 : 144;
    if (qt == MLQ_Q4_K && down) bytes = 144;
    if (qt == MLQ_Q5_K) bytes = 176;
    if (qt == MLQ_Q6_K) bytes = 210;
    return (long long)rows * (cols / 256) * bytes;
}

// Bytes the kernels read from an expert tensor: E experts at `stride` apart, each
// rows x row_bytes (the two differ only under the reference's stride rule).
static size_t expert_extent(long long stride, int E, int qt, int rows, int cols) {
    const size_t mat = (size_t)rows * mlq_row_bytes(qt, cols);
    const size_t a = (size_t)stride * E, b = (size_t)stride * (E - 1) + mat;
    return a > b ? a : b;
}

static bool build_plan(const BC *c, CallScope &cs, ModelPlan &P) {
    const int L = c->L, N = c->N, NH = c->NH, NKH = c->NKH, HD = c->HD, inner = NH * HD;
    P.layers.assign(L, LayerPlan{});
    const std::vector<int> win = windows_of(c);
    for (int l = 0; l < L; l++) {
        LayerPlan &lp = P.layers[l];
        lp.window = l < (int)win.size() ? win[l] : 0;
        lp.an = Fv(cs, c->wAN ? c->wAN[l] : nullptr, N);
        lp.fn = Fv(cs, c->wFN ? c->wFN[l] : nullptr, N);
        lp.ssm = c->layer_types && c->layer_types[l] == 1 && c->ssm_conv1d && c->ssm_conv1d[l];
        if (c->wAttnG && c->wAttnG[l]) {
            lp.qattng = at(c->attnG_quant, l, 8);
            lp.wattng = lp.ssm ? W(cs, c->wAttnG[l], lp.qattng, inner, N) : W(cs, c->wAttnG[l], lp.qattng, N, inner);
        }
        if (lp.ssm) {
            lp.conv = Fv(cs, c->ssm_conv1d[l], (size_t)2 * inner);
            lp.ssm_a = Fv(cs, c->ssm_a ? c->ssm_a[l] : nullptr, kSsmGroups);
            lp.ssm_dt = Fv(cs, c->ssm_dt_bias ? c->ssm_dt_bias[l] : nullptr, kSsmGroups);
            lp.ssm_alpha = Fv(cs, c->ssm_alpha ? c->ssm_alpha[l] : nullptr, (size_t)kSsmGroups * kSsmDtRank);
            lp.ssm_beta = Fv(cs, c->ssm_beta ? c->ssm_beta[l] : nullptr, (size_t)kSsmGroups * kSsmDtRank);
            if (c->wSsmOut && c->wSsmOut[l]) {
                lp.qssmout = at(c->ssm_out_quant, l, 8);
                lp.wssmout = W(cs, c->wSsmOut[l], lp.qssmout, N, inner);
            }
            if (!lp.ssm_a || !lp.ssm_dt || !lp.ssm_alpha || !lp.ssm_beta) {
                set_error(MLQ_ERR_ARG, "batch_forward: SSM layer %d without its parameters", l);
                return false;
            }
        } else {
            lp.nq = at(c->nQ, l, inner);
            lp.nk = at(c->nK, l, NKH * HD);
            lp.nv = at(c->nV, l, NKH * HD);
            lp.no = at(c->nO, l, N);
            // the reference reads Q, K, V rows at b*NH*HD / b*NKH*HD and o-proj rows at b*N
            if (lp.nq != inner || lp.nk != NKH * HD || lp.nv != NKH * HD || lp.no != N || NKH * HD > N) {
                set_error(MLQ_ERR_ARG, "batch_forward: layer %d projection sizes %d/%d/%d/%d do not match NH*HD, "
                                       "NKH*HD, N", l, lp.nq, lp.nk, lp.nv, lp.no);
                return false;
            }
            if (c->wQKV && c->wQKV[l]) {
                lp.qqkv = at(c->qkv_quant, l, 8);
                lp.wqkv = W(cs, c->wQKV[l], lp.qqkv, inner + 2 * N, c->nc);
            } else if (c->wQK && c->wQK[l]) {
                lp.qqk = at(c->qk_quant, l, 8);
                lp.wqk = W(cs, c->wQK[l], lp.qqk, lp.nq + lp.nk, c->nc);
                lp.qv = at(c->v_quant, l, 8);
                lp.wv = W(cs, c->wV[l], lp.qv, lp.nv, c->nc);
            } else {
                lp.qq = at(c->q_quant, l, 8);
                lp.qk = at(c->k_quant, l, 8);
                lp.qv = at(c->v_quant, l, 8);
                lp.wq = W(cs, c->wQ ? c->wQ[l] : nullptr, lp.qq, lp.nq, c->nc);
                lp.wk = W(cs, c->wK ? c->wK[l] : nullptr, lp.qk, lp.nk, c->nc);
                lp.wv = W(cs, c->wV ? c->wV[l] : nullptr, lp.qv, lp.nv, c->nc);
                if (!lp.wq || !lp.wk || !lp.wv) {
                    set_error(MLQ_ERR_ARG, "batch_forward: attention layer %d without Q/K/V weights", l);
                    return false;
                }
            }
            if (!lp.wattng) {
                lp.qo = at(c->o_quant, l, 8);
                lp.wo = W(cs, c->wO ? c->wO[l] : nullptr, lp.qo, lp.no, inner);
                if (!lp.wo) {
                    set_error(MLQ_ERR_ARG, "batch_forward: attention layer %d without an output projection", l);
                    return false;
                }
            }
        }
        if (c->n_experts > 0 && c->n_experts_per_tok > 0) {
            const int E = c->n_experts, M = c->moe_intermediate;
            lp.router = Fv(cs, c->w_gate_inp ? c->w_gate_inp[l] : nullptr, (size_t)E * N);
            lp.gstride = expert_stride(c->gate_exp_quant, M, N, false);
            lp.ustride = expert_stride(c->up_exp_quant, M, N, false);
            lp.dstride = expert_stride(c->down_exp_quant, N, M, true);
            if (!lp.router || !lp.gstride || !lp.ustride || !lp.dstride || !c->w_gate_exps || !c->w_up_exps ||
                !c->w_down_exps) {
                set_error(MLQ_ERR_ARG, "batch_forward: MoE layer %d incomplete", l);
                return false;
            }
            lp.gexp = (const uint8_t *)cs.weights(c->w_gate_exps[l], expert_extent(lp.gstride, E, c->gate_exp_quant, M, N));
            lp.uexp = (const uint8_t *)cs.weights(c->w_up_exps[l], expert_extent(lp.ustride, E, c->up_exp_quant, M, N));
            lp.dexp = (const uint8_t *)cs.weights(c->w_down_exps[l], expert_extent(lp.dstride, E, c->down_exp_quant, N, M));
            if (c->wSHexpG && c->wSHexpG[l]) {
                lp.qshg = at(c->shexp_g_quant, l, 8);
                lp.qshu = at(c->shexp_u_quant, l, 8);
                lp.qshd = at(c->shexp_d_quant, l, 8);
                lp.shg = W(cs, c->wSHexpG[l], lp.qshg, kShexpFF, N);
                lp.shu = W(cs, c->wSHexpU[l], lp.qshu, kShexpFF, N);
                lp.shd = W(cs, c->wSHexpD[l], lp.qshd, N, kShexpFF);
                lp.shrouter = Fv(cs, c->wShexpRouter ? c->wShexpRouter[l] : nullptr, N);
            }
        } else if (c->wG && c->wG[l]) {
            lp.qg = at(c->g_quant, l, 8);
            lp.qu = at(c->u_quant, l, 8);
            lp.qd = at(c->d_quant, l, 8);
            lp.ng = at(c->nG, l, c->FF);
            lp.nu = at(c->nU, l, c->FF);
            lp.nd = at(c->nD, l, N);
            lp.wg = W(cs, c->wG[l], lp.qg, lp.ng, c->nc);
            lp.wu = W(cs, c->wU[l], lp.qu, lp.nu, c->nc);
            lp.wd = W(cs, c->wD[l], lp.qd, lp.nd, c->FF);
        }
        if (cs.failed) return false;
    }
    const int rope_dim = c->rope_dim > 0 ? c->rope_dim : HD;
    P.emb = (const float *)cs.weights(c->emb, embed_bytes(c->emb_quant, N, c->V));
    P.onw = Fv(cs, c->onw, N);
    P.wout = W(cs, c->wOut, c->outQuant, c->outNR, c->outNC);
    P.cos_t = Fv(cs, c->cos_table, (size_t)c->max_ctx * (rope_dim / 2));
    P.sin_t = Fv(cs, c->sin_table, (size_t)c->max_ctx * (rope_dim / 2));
    return !cs.failed && P.emb && P.wout && P.cos_t && P.sin_t;
}

static int fwd_fail(CallScope &cs, int rc) {
    cs.failed = true;
    cs.finish();
    return rc;
}

// ------------------------------------------------------------------------------ step buffers
struct StepDims {
    int B, N, inner, kvrow, FF, E, topk, M, outNR, NH, HD, L;
    bool ssm;
    int gq = 0, uq = 0, dq = 0;   // routed expert types (grouped expert scratch)
};

// routed experts run through the grouped expert GEMV when its tilings cover their types
static bool moe_grouped_ok(const StepDims &d) {
    return d.E > 0 && d.topk > 0 && d.M > 0 && d.N % 32 == 0 && d.M % 32 == 0 && d.E <= 1024 &&
           grouped_tiles_per_expert(d.gq, d.M, d.N) && grouped_tiles_per_expert(d.uq, d.M, d.N) &&
           grouped_tiles_per_expert(d.dq, d.N, d.M) && !getenv("MLQ_NO_GROUPED_MOE");
}

// Device buffers of one decode step.  The head (pos, len, KV pointer arrays, page tables)
// is one contiguous block so the per-step host inputs go up in one copy.
struct StepBufs {
    uint8_t *head = nullptr;
    size_t head_fixed = 0;   // bytes before the page tables
    int *pos = nullptr, *len = nullptr, *tab = nullptr;
    float **pools = nullptr, **mk = nullptr, **mv = nullptr;
    int *tok = nullptr, *e_idx = nullptr;
    float *xin = nullptr, *x = nullptr, *xn = nullptr, *res = nullptr, *qkv = nullptr, *q = nullptr, *k = nullptr,
          *v = nullptr, *att = nullptr, *tmp = nullptr, *g = nullptr, *u = nullptr, *h = nullptr, *logits_e = nullptr,
          *e_w = nullptr, *hm = nullptr, *hm2 = nullptr, *score = nullptr, *attn_scr = nullptr, *hfin = nullptr,
          *logits = nullptr, *state = nullptr;
    uint8_t *px = nullptr, *pa = nullptr, *ph = nullptr;   // packed activation rows (decode GEMV inputs)
    size_t attn_sb = 0;
    MoeGroupedScratch moe{};   // grouped routed experts (when moe_grouped_ok)
    float *y_moe = nullptr;    // [B * topk][N] expert outputs before the weighted combine
};

static size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

// lay the buffers out from base (base == nullptr: only count); returns the bytes used
static size_t carve(StepBufs &b, uint8_t *base, const StepDims &d) {
    size_t o = 0;
    auto take = [&](size_t bytes) -> uint8_t * {
        uint8_t *p = base ? base + o : nullptr;
        o += al256(bytes);
        return p;
    };
    const size_t B = d.B;
    // head: pos[B] len[B] | pools[B] mk[B] mv[B] | tab[B][1024]
    b.head = base ? base : nullptr;
    const size_t ints = 2 * B * sizeof(int);
    const size_t ptr_off = (ints + 15) & ~(size_t)15;
    b.head_fixed = ptr_off + 3 * B * sizeof(float *);
    uint8_t *h = take(b.head_fixed + B * 1024 * sizeof(int));
    if (h) {
        b.pos = (int *)h;
        b.len = b.pos + B;
        b.pools = (float **)(h + ptr_off);
        b.mk = b.pools + B;
        b.mv = b.mk + B;
        b.tab = (int *)(h + b.head_fixed);
    }
    const int FFmax = d.FF > kShexpFF ? d.FF : kShexpFF;
    const int wide = FFmax > d.inner ? FFmax : d.inner;
    const int qkv_w = d.inner + 2 * (d.N > d.kvrow ? d.N : d.kvrow);
    const int tk = d.topk > 0 ? d.topk : 1, M = d.M > 0 ? d.M : 1;
    b.tok = (int *)take(B * sizeof(int));
    b.xin = (float *)take(B * d.N * 4);
    b.x = (float *)take(B * d.N * 4);
    b.xn = (float *)take(B * d.N * 4);
    b.res = (float *)take(B * d.N * 4);
    b.qkv = (float *)take(B * (size_t)(qkv_w > d.N ? qkv_w : d.N) * 4);
    b.q = (float *)take(B * d.inner * 4);
    b.k = (float *)take(B * d.kvrow * 4);
    b.v = (float *)take(B * d.kvrow * 4);
    b.att = (float *)take(B * d.inner * 4);
    b.tmp = (float *)take(B * (size_t)(d.inner > d.N ? d.inner : d.N) * 4);
    b.g = (float *)take(B * (size_t)wide * 4);
    b.u = (float *)take(B * (size_t)wide * 4);
    b.h = (float *)take(B * (size_t)wide * 4);
    b.logits_e = (float *)take(B * (size_t)(d.E > 0 ? d.E : 1) * 4);
    b.e_idx = (int *)take(B * tk * sizeof(int));
    b.e_w = (float *)take(B * tk * 4);
    b.hm = (float *)take(B * (size_t)tk * M * 4);
    b.hm2 = (float *)take(B * (size_t)tk * M * 4);
    b.score = (float *)take(B * 4);
    b.attn_sb = attn_scratch_bytes(d.B, d.NH, d.HD);
    b.attn_scr = (float *)take(b.attn_sb);
    b.hfin = (float *)take(B * d.N * 4);
    b.logits = (float *)take(B * (size_t)d.outNR * 4);
    b.state = d.ssm ? (float *)take((size_t)d.L * kSsmGroups * kSsmState * 4) : nullptr;
    b.px = take(packed_rows_bytes(d.B, d.N));
    b.pa = take(packed_rows_bytes(d.B, d.inner));
    b.ph = take(packed_rows_bytes(d.B, wide));
    if (moe_grouped_ok(d)) {
        const int R = d.B * d.topk;
        uint8_t *m = take(moe_grouped_scratch_bytes(d.gq, d.uq, d.dq, R, d.E, d.M, d.N));
        if (m) moe_grouped_carve(b.moe, m, d.gq, d.uq, d.dq, R, d.E, d.M, d.N);
        b.y_moe = (float *)take((size_t)R * d.N * 4);
    }
    return o;
}

static size_t step_bytes(const StepDims &d) {
    StepBufs tmp;
    return carve(tmp, nullptr, d);
}

static int max_blocks_used(const std::vector<int> &pos, int ps) {
    int m = 0;
    for (int p : pos) m = p / ps + 1 > m ? p / ps + 1 : m;
    return m;
}

// positions, lengths, KV pointer arrays and page tables (row stride tab_w) in one copy
static int upload_step_inputs(const StepBufs &sb, const StepDims &d, const std::vector<int> &pos,
                              const std::vector<int> &lens, const std::vector<int> &tables,
                              const std::vector<float *> &pools, const std::vector<float *> &mk,
                              const std::vector<float *> &mv, int tab_w, cudaStream_t s) {
    const int B = d.B;
    std::vector<uint8_t> host(sb.head_fixed + (size_t)B * tab_w * sizeof(int));
    int *hp = (int *)host.data();
    memcpy(hp, pos.data(), B * sizeof(int));
    memcpy(hp + B, lens.data(), B * sizeof(int));
    uint8_t *ptrs = host.data() + ((uint8_t *)sb.pools - sb.head);
    memcpy(ptrs, pools.data(), B * sizeof(float *));
    memcpy(ptrs + B * sizeof(float *), mk.data(), B * sizeof(float *));
    memcpy(ptrs + 2 * B * sizeof(float *), mv.data(), B * sizeof(float *));
    int *ht = (int *)(host.data() + sb.head_fixed);
    for (int b = 0; b < B; b++) memcpy(ht + (size_t)b * tab_w, &tables[(size_t)b * 1024], tab_w * sizeof(int));
    return MLQ_CUDA(cudaMemcpyAsync(sb.head, host.data(), host.size(), cudaMemcpyHostToDevice, s)) ? MLQ_OK
                                                                                                : MLQ_ERR_CUDA;
}

// Every device launch of one step.  tab_w: page-table row stride in sb.tab; attn_len: the
// length the attention splits are planned for (>= every sequence's length); h_tok: host
// token ids (only the per-row Q4_K embedding decode reads them).
static int enqueue_step(const BC *c, const ModelPlan *P, const StepBufs &sb, const StepDims &d, bool compat,
                        int attn_len, int tab_w, const int *d_tok, const int *h_tok, const float *xin, float *d_state,
                        float *hfin, float *d_logits, cudaStream_t s) {
    const int B = d.B, N = d.N, inner = d.inner, kvrow = d.kvrow, NH = c->NH, NKH = c->NKH, HD = c->HD, L = d.L;
    const int rope_dim = c->rope_dim > 0 ? c->rope_dim : HD;
    const int topk = d.topk, M = d.M;
    const MlqKVBlock *kv0 = c->kv_array[0];
    float *x = sb.x, *xn = sb.xn, *res = sb.res, *qkv = sb.qkv, *q = sb.q, *k = sb.k, *v = sb.v, *att = sb.att,
          *tmp = sb.tmp, *g = sb.g, *u = sb.u, *h = sb.h;
    int rc = MLQ_OK;
#define MLQ_TRY(expr)                  \
    do {                               \
        if (rc == MLQ_OK) rc = (expr); \
    } while (0)
    MLQ_TRY(launch_embed(P->emb, c->emb_quant, d_tok, h_tok, x, B, N, c->V, s));
    const int ps = kv0->pt.page_size;
    const long long layer_stride = (long long)kv0->pt.n_pages * ps * kvrow;
    const float scale = 1.0f / sqrtf((float)HD);
    // norm output and projection input: xn / xn normally; x / the workspace's xn region in
    // reference-compatibility mode
    float *nout = compat ? x : xn;
    const float *pin = compat ? xin : xn;
    const float inf = HUGE_VALF;
    // Decode path (B <= 8, outside compatibility mode): every RMSNorm also writes its rows
    // as packed activation rows, and the projections run as segmented decode GEMVs on them
    // (Q/K/V of one type in one launch, gate/up with the SiLU-mul, o/down with the residual
    // add); a shape the decode GEMV does not take falls back to the plain GEMV.
    const bool fast = !compat && B <= 8 && N % 32 == 0 && inner % 32 == 0 && c->FF % 32 == 0 &&
                      !getenv("MLQ_NO_DECODE_GEMV");
    auto norm = [&](const float *w, float *out_fp32) -> int {
        if (fast && launch_rms_norm_encode(out_fp32, x, w, res, B, N, c->eps, 1, sb.px, s) == MLQ_OK) return MLQ_OK;
        return launch_rms_norm(out_fp32, x, w, res, B, N, c->eps, 1, s);
    };
    // seg GEMV over n matrices sharing input planes; false: not taken (caller falls back)
    auto seg = [&](int qt, int n, const uint8_t *const *W, const int *rows, float *const *out, const float *const *rs,
                   int pair, const uint8_t *planes, int K) -> bool {
        if (!fast || rc != MLQ_OK) return false;
        const int r2 = launch_gemv_seg(qt, n, W, rows, out, rs, pair, planes, B, K, s);
        if (r2 == MLQ_ERR_UNSUPPORTED) return false;
        rc = r2;
        return true;
    };
    for (int l = 0; l < L && rc == MLQ_OK; l++) {
        const LayerPlan &lp = P->layers[l];
        MLQ_TRY(norm(lp.an, nout));
        if (lp.ssm) {
            float *st = d_state + (size_t)l * kSsmGroups * kSsmState;
            MLQ_TRY(launch_ssm_decode_step(pin, att, lp.conv, lp.ssm_a, lp.ssm_dt, lp.ssm_alpha, lp.ssm_beta, st, B, N,
                                           inner, kSsmGroups, kSsmState, kSsmDtRank, s));
            if (lp.wattng) {
                MLQ_TRY(launch_matmul(lp.wattng, lp.qattng, pin, g, inner, N, B, 0, s));
                MLQ_TRY(launch_mul(att, g, (long long)B * inner, s));
            } else {
                cudaMemsetAsync(att, 0, sizeof(float) * (size_t)B * inner, s);
            }
            if (lp.wssmout) {
                MLQ_TRY(launch_matmul(lp.wssmout, lp.qssmout, att, tmp, N, inner, B, 0, s));
                MLQ_TRY(launch_add(x, res, tmp, (long long)B * N, s));
            } else {
                cudaMemcpyAsync(x, res, sizeof(float) * (size_t)B * N, cudaMemcpyDeviceToDevice, s);
            }
        } else {
            if (lp.wqkv) {
                const int n_qkv = inner + 2 * N;
                MLQ_TRY(launch_matmul(lp.wqkv, lp.qqkv, pin, qkv, n_qkv, c->nc, B, 0, s));
                k_copy_cols<<<dim3(grid1(inner) > 16 ? 16 : grid1(inner), B), 256, 0, s>>>(q, qkv, inner,
                                                                                        compat ? inner : n_qkv, 0);
                k_copy_cols<<<dim3(grid1(kvrow) > 16 ? 16 : grid1(kvrow), B), 256, 0, s>>>(k, qkv, kvrow, n_qkv, inner);
                k_copy_cols<<<dim3(grid1(kvrow) > 16 ? 16 : grid1(kvrow), B), 256, 0, s>>>(v, qkv, kvrow, n_qkv,
                                                                                        inner + N);
                count_launch(3);
            } else if (lp.wqk) {
                const int nqk = lp.nq + lp.nk;
                MLQ_TRY(launch_matmul(lp.wqk, lp.qqk, pin, qkv, nqk, c->nc, B, 0, s));
                k_copy_cols<<<dim3(grid1(inner) > 16 ? 16 : grid1(inner), B), 256, 0, s>>>(q, qkv, inner,
                                                                                        compat ? inner : nqk, 0);
                k_copy_cols<<<dim3(grid1(kvrow) > 16 ? 16 : grid1(kvrow), B), 256, 0, s>>>(k, qkv, kvrow, nqk, lp.nq);
                count_launch(2);
                MLQ_TRY(launch_matmul(lp.wv, lp.qv, pin, v, lp.nv, c->nc, B, 0, s));
            } else {
                // Q, K, V grouped by type into decode GEMV launches
                const uint8_t *Wm[3] = {lp.wq, lp.wk, lp.wv};
                const int qts[3] = {lp.qq, lp.qk, lp.qv}, rows[3] = {lp.nq, lp.nk, lp.nv};
                float *outs[3] = {q, k, v};
                bool done[3] = {false, false, false};
                for (int i = 0; i < 3 && fast && c->nc == N; i++) {
                    if (done[i]) continue;
                    const uint8_t *gw[3];
                    int gr[3], n = 0;
                    float *go[3];
                    int idx[3];
                    for (int j = i; j < 3; j++)
                        if (!done[j] && qts[j] == qts[i]) {
                            gw[n] = Wm[j]; gr[n] = rows[j]; go[n] = outs[j]; idx[n++] = j;
                        }
                    if (seg(qts[i], n, gw, gr, go, nullptr, 0, sb.px, N))
                        for (int j = 0; j < n; j++) done[idx[j]] = true;
                }
                for (int i = 0; i < 3; i++)
                    if (!done[i]) MLQ_TRY(launch_matmul(Wm[i], qts[i], pin, outs[i], rows[i], c->nc, B, 0, s));
            }
            KVView kv{nullptr, nullptr, sb.tab, tab_w, (long long)ps * kvrow, ps, kvrow, sb.pools, layer_stride, l,
                      kv0->pt._n_layers};
            kv.n_pages = kv0->pt.n_pages;
            // the attention output also as packed rows for the o projection (decode path)
            const bool o_fast = fast && !lp.wattng && lp.no == N;
            const bool att_packed = o_fast && inner == NH * HD && attn_packs_output(NH, NKH, HD);
            // RoPE + KV store (+ KVBlock mirror) inside the attention kernel when the row layout
            // allows; otherwise in one launch before it, or as separate steps
            bool attn_done = false;
            if (rc == MLQ_OK && inner == NH * HD && kvrow == NKH * HD && !getenv("MLQ_NO_ATTN_ROPE")) {
                AttnRope ar;
                ar.pos = sb.pos;
                ar.cos_t = P->cos_t;
                ar.sin_t = P->sin_t;
                ar.rope_dim = rope_dim;
                ar.k_new = k;
                ar.v_new = v;
                ar.mk = sb.mk;
                ar.mv = sb.mv;
                const int ra = launch_attn_decode(q, kv, sb.len, 0, attn_len, B, NH, NKH, HD, lp.window, scale, att,
                                                  sb.attn_scr, sb.attn_sb, s, att_packed ? sb.pa : nullptr, &ar);
                if (ra != MLQ_ERR_UNSUPPORTED) {
                    rc = ra;
                    attn_done = true;
                }
            }
            if (!attn_done) {
                const bool fused_kv = rc == MLQ_OK && inner == NH * HD && kvrow == NKH * HD &&
                                      launch_rope_kv(q, k, v, B, NH, NKH, HD, rope_dim, sb.pos, P->cos_t, P->sin_t,
                                                     kv, sb.mk, sb.mv, s) == MLQ_OK;
                if (!fused_kv) {
                    MLQ_TRY(launch_rope_neox(q, B, inner, NH, HD, sb.pos, 0, P->cos_t, P->sin_t, rope_dim, s));
                    MLQ_TRY(launch_rope_neox(k, B, kvrow, NKH, HD, sb.pos, 0, P->cos_t, P->sin_t, rope_dim, s));
                    MLQ_TRY(launch_kv_write(kv, nullptr, nullptr, k, v, sb.pos, 0, B, kvrow, s));
                    if (rc == MLQ_OK) {
                        k_kv_mirror<<<dim3(grid1(kvrow) > 16 ? 16 : grid1(kvrow), B), 256, 0, s>>>(
                            sb.mk, sb.mv, sb.tab, tab_w, sb.pos, k, v, kvrow, ps, l);
                        count_launch();
                    }
                }
                MLQ_TRY(launch_attn_decode(q, kv, sb.len, 0, attn_len, B, NH, NKH, HD, lp.window, scale, att,
                                           sb.attn_scr, sb.attn_sb, s, att_packed ? sb.pa : nullptr));
            }
            bool o_done = false;
            if (o_fast && rc == MLQ_OK) {   // x = res + W_o att
                if (!att_packed) MLQ_TRY(launch_encode_packed(att, nullptr, nullptr, B, inner, sb.pa, s));
                const uint8_t *wo = lp.wo;
                const int no = lp.no;
                float *xo = x;
                const float *ro = res;
                o_done = seg(lp.qo, 1, &wo, &no, &xo, &ro, 0, sb.pa, inner);
            }
            if (!o_done) {
                if (lp.wattng) MLQ_TRY(launch_matmul(lp.wattng, lp.qattng, att, tmp, N, inner, B, 0, s));
                else MLQ_TRY(launch_matmul(lp.wo, lp.qo, att, tmp, lp.no, inner, B, 0, s));
                MLQ_TRY(launch_add(x, res, tmp, (long long)B * N, s));
            }
        }
        MLQ_TRY(norm(lp.fn, nout));
        if (lp.router) {
            const int E = c->n_experts;
            MLQ_TRY(launch_matmul((const uint8_t *)lp.router, MLQ_F32, pin, sb.logits_e, E, N, B, 0, s));
            MLQ_TRY(launch_router_topk(sb.logits_e, B, E, topk, 0, sb.e_idx, sb.e_w, s));
            if (sb.y_moe) {
                // every active expert streamed once for all of its (token, slot) rows, then
                // x = res + sum_i w_i y_i in slot order
                MLQ_TRY(launch_moe_grouped(c->gate_exp_quant, c->up_exp_quant, c->down_exp_quant, lp.gexp, lp.uexp,
                                           lp.dexp, lp.gstride, lp.ustride, lp.dstride, E, sb.e_idx, B * topk, topk,
                                           M, N, pin, sb.y_moe, inf, sb.moe, s));
                MLQ_TRY(launch_ep_combine(sb.y_moe, nullptr, sb.e_w, B, topk, N, res, x, s));
            } else {
                MLQ_TRY(launch_moe_experts(c->gate_exp_quant, c->up_exp_quant, c->down_exp_quant, lp.gexp, lp.uexp,
                                           lp.dexp, lp.gstride, lp.ustride, lp.dstride, sb.e_idx, sb.e_w, topk, B, M,
                                           N, pin, sb.hm, sb.hm2, x, res, inf, s));
            }
            if (lp.shg && lp.shrouter) {
                k_dot_rows<<<B, 256, 0, s>>>(pin, lp.shrouter, sb.score, N);
                count_launch();
                MLQ_TRY(launch_matmul(lp.shg, lp.qshg, pin, g, kShexpFF, N, B, 0, s));
                MLQ_TRY(launch_matmul(lp.shu, lp.qshu, pin, u, kShexpFF, N, B, 0, s));
                k_shexp_act<<<grid1((long long)B * kShexpFF), 256, 0, s>>>(h, g, u, (long long)B * kShexpFF);
                count_launch();
                MLQ_TRY(launch_matmul(lp.shd, lp.qshd, h, tmp, N, kShexpFF, B, 0, s));
                k_add_scaled_pos<<<dim3(grid1(N) > 16 ? 16 : grid1(N), B), 256, 0, s>>>(x, tmp, sb.score, N);
                count_launch();
            }
        } else if (lp.wg) {
            bool h_done = false;
            if (lp.qg == lp.qu && lp.ng == lp.nu && lp.ng == c->FF && c->nc == N) {   // h = silu(W_g x) * (W_u x)
                const uint8_t *gu[2] = {lp.wg, lp.wu};
                const int rows[2] = {lp.ng, lp.nu};
                float *ho[2] = {h, h};
                h_done = seg(lp.qg, 2, gu, rows, ho, nullptr, 1, sb.px, N);
            }
            if (!h_done) {
                MLQ_TRY(launch_matmul(lp.wg, lp.qg, pin, g, lp.ng, c->nc, B, 0, s));
                MLQ_TRY(launch_matmul(lp.wu, lp.qu, pin, u, lp.nu, c->nc, B, 0, s));
                k_silu_mul<<<grid1((long long)B * c->FF), 256, 0, s>>>(h, g, u, (long long)B * c->FF);
                count_launch();
            }
            bool d_done = false;
            if (fast && lp.nd == N && rc == MLQ_OK) {   // x = res + W_d h
                MLQ_TRY(launch_encode_packed(h, nullptr, nullptr, B, c->FF, sb.ph, s));
                const uint8_t *wd = lp.wd;
                const int nd = lp.nd;
                float *xo = x;
                const float *ro = res;
                d_done = seg(lp.qd, 1, &wd, &nd, &xo, &ro, 0, sb.ph, c->FF);
            }
            if (!d_done) {
                MLQ_TRY(launch_matmul(lp.wd, lp.qd, h, tmp, lp.nd, c->FF, B, 0, s));
                MLQ_TRY(launch_add(x, res, tmp, (long long)B * N, s));
            }
        } else if (!compat) {
            cudaMemcpyAsync(x, res, sizeof(float) * (size_t)B * N, cudaMemcpyDeviceToDevice, s);
        }   // (with no FFN the reference leaves the normalised activations in x)
    }
    // the final normalised hidden state also lands in ws[0 : B*N], where the reference
    // leaves it (its x buffer is the start of the workspace)
    MLQ_TRY(norm(P->onw, hfin));
    {
        const uint8_t *wout = P->wout;
        const int nr = c->outNR;
        float *lo = d_logits;
        if (!(c->outNC == N && seg(c->outQuant, 1, &wout, &nr, &lo, nullptr, 0, sb.px, N)))
            MLQ_TRY(launch_matmul(P->wout, c->outQuant, hfin, d_logits, c->outNR, c->outNC, B, 0, s));
    }
#undef MLQ_TRY
    return rc;
}

// ------------------------------------------------------------------------------ CUDA graphs
// A step is captured once per (plan, batch size, attention-length bucket, mode) and
// replayed; the per-step inputs (positions, page tables, KV pointers, tokens, the
// compatibility-mode projection input, a host SSM state) are copied into the graph's own
// buffers before the replay and its outputs copied out after it.  Attention splits are
// planned for the bucket (a power of two >= the longest sequence), the kernels read each
// sequence's own length, so one graph serves every step inside the bucket.
struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    uint8_t *mem = nullptr;
    StepBufs sb;
    unsigned long long launches = 0;
};
struct GraphKey {
    int dev;
    uintptr_t bc;
    unsigned long long gen;
    int B, bucket, tab_w, compat, state_dev, ws_out;
    uintptr_t state_ptr;
    bool operator<(const GraphKey &o) const {
        return std::tie(dev, bc, gen, B, bucket, tab_w, compat, state_dev, ws_out, state_ptr) <
               std::tie(o.dev, o.bc, o.gen, o.B, o.bucket, o.tab_w, o.compat, o.state_dev, o.ws_out, o.state_ptr);
    }
};
static std::mutex g_graph_mu;
static std::map<GraphKey, GraphEntry> g_graphs;
static std::map<GraphKey, bool> g_graph_failed;
static std::map<GraphKey, bool> g_graph_seen;

static bool graphs_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("MLQ_NO_GRAPHS");
        v = (e && atoi(e) != 0) ? 0 : 1;
    }
    return v == 1;
}

// the legacy default stream cannot be captured
static bool capturable(cudaStream_t s) { return s != nullptr && s != cudaStreamLegacy; }

static void destroy_graphs() {
    std::lock_guard<std::mutex> lk(g_graph_mu);
    for (auto &kv : g_graphs) {
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
        if (kv.second.mem) cudaFree(kv.second.mem);
    }
    g_graphs.clear();
    g_graph_failed.clear();
    g_graph_seen.clear();
}

static int run_graph_step(const BC *c, const ModelPlan *P, const StepDims &d, bool compat, const std::vector<int> &pos,
                          const std::vector<int> &lens, const std::vector<int> &tables,
                          const std::vector<float *> &pools, const std::vector<float *> &mk,
                          const std::vector<float *> &mv, int tab_w_used, int max_len, const int *tokens,
                          const float *ws_xn, float *ws, cudaStream_t s) {
    Ctx *cx = ctx();
    if (!cx) return mlq_last_error();
    const MlqKVBlock *kv0 = c->kv_array[0];
    int bucket = 64;
    while (bucket < max_len) bucket *= 2;
    int tab_w = (bucket + kv0->pt.page_size - 1) / kv0->pt.page_size;
    if (tab_w > 1024) tab_w = 1024;
    if (tab_w < tab_w_used) tab_w = tab_w_used;
    const bool state_dev = d.ssm && is_device_ptr(c->ssm_state);
    GraphKey key{cx->device, (uintptr_t)c, P->gen, d.B, bucket, tab_w, compat ? 1 : 0, state_dev ? 1 : 0,
                 ws ? 1 : 0, state_dev ? (uintptr_t)c->ssm_state : 0};
    std::lock_guard<std::mutex> lk(g_graph_mu);
    if (g_graph_failed.count(key)) return MLQ_ERR_UNSUPPORTED;
    auto it = g_graphs.find(key);
    if (it == g_graphs.end() && !g_graph_seen.count(key)) {
        // the first step of a shape runs eagerly (one-time kernel attributes, lazy state)
        g_graph_seen[key] = true;
        return MLQ_ERR_UNSUPPORTED;
    }
    if (it == g_graphs.end()) {
        GraphEntry e;
        const size_t bytes = step_bytes(d);
        if (!MLQ_CUDA(cudaMalloc(&e.mem, bytes))) return MLQ_ERR_CUDA;
        carve(e.sb, e.mem, d);
        float *dstate = d.ssm ? (state_dev ? c->ssm_state : e.sb.state) : nullptr;
        // capture (nothing executes); zero host ids: the graph path never decodes Q4_K rows
        std::vector<int> h_tok(d.B, 0);
        const unsigned long long l0 = mlq_launch_count();
        cudaGraph_t graph = nullptr;
        int rc = MLQ_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal)) ? MLQ_OK : MLQ_ERR_CUDA;
        if (rc == MLQ_OK) {
            rc = enqueue_step(c, P, e.sb, d, compat, bucket, tab_w, e.sb.tok, h_tok.data(), e.sb.xin, dstate,
                              e.sb.hfin, e.sb.logits, s);
            const cudaError_t ce = cudaStreamEndCapture(s, &graph);
            if (ce != cudaSuccess) {
                cudaGetLastError();
                if (rc == MLQ_OK) rc = MLQ_ERR_UNSUPPORTED;
            }
        }
        if (rc == MLQ_OK && graph) {
            if (cudaGraphInstantiate(&e.exec, graph, 0) != cudaSuccess) {
                cudaGetLastError();
                rc = MLQ_ERR_UNSUPPORTED;
            }
        }
        if (graph) cudaGraphDestroy(graph);
        e.launches = mlq_launch_count() - l0;
        if (rc != MLQ_OK) {
            cudaFree(e.mem);
            g_graph_failed[key] = true;
            cudaGetLastError();
            return MLQ_ERR_UNSUPPORTED;
        }
        it = g_graphs.emplace(key, e).first;
    } else {
        count_launch((int)it->second.launches);
    }
    GraphEntry &e = it->second;
    const StepDims &dd = d;
    int rc = upload_step_inputs(e.sb, dd, pos, lens, tables, pools, mk, mv, tab_w, s);
    bool host_io = false;
    auto cp = [&](void *dst, const void *src, size_t bytes) {
        if (rc != MLQ_OK) return;
        if (!is_device_ptr(dst) || !is_device_ptr(src)) host_io = true;
        if (!MLQ_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s))) rc = MLQ_ERR_CUDA;
    };
    cp(e.sb.tok, tokens, sizeof(int) * d.B);
    if (compat) cp(e.sb.xin, ws_xn, sizeof(float) * (size_t)d.B * d.N);
    const size_t state_bytes = sizeof(float) * (size_t)d.L * kSsmGroups * kSsmState;
    if (d.ssm && !state_dev) cp(e.sb.state, c->ssm_state, state_bytes);
    if (rc == MLQ_OK && !MLQ_CUDA(cudaGraphLaunch(e.exec, s))) rc = MLQ_ERR_CUDA;
    cp(c->logits, e.sb.logits, sizeof(float) * (size_t)d.B * d.outNR);
    if (ws) cp(ws, e.sb.hfin, sizeof(float) * (size_t)d.B * d.N);
    if (d.ssm && !state_dev) cp(c->ssm_state, e.sb.state, state_bytes);
    if (rc == MLQ_OK && host_io && !MLQ_CUDA(cudaStreamSynchronize(s))) rc = MLQ_ERR_CUDA;
    return rc;
}

}  // namespace mlq

using namespace mlq;

extern "C" {

size_t mlq_sizeof_bc(void) { return sizeof(BC); }

// Sliding-window attention per layer for batch_forward on this model description: layer l
// attends to its last windows[l] positions (0 = all of them).  The reference's engine has no
// windowed attention; GPT-OSS-style models alternate full and 128-token windows.  The setting
// belongs to the BC address; windows == NULL or L == 0 clears it.
int mlq_set_attention_windows(const void *bc, const int *windows, int L) {
    if (!bc || L < 0 || (L > 0 && !windows)) {
        set_error(MLQ_ERR_ARG, "mlq_set_attention_windows: null model or windows");
        return MLQ_ERR_ARG;
    }
    for (int l = 0; l < L; l++) {
        if (windows[l] < 0) {
            set_error(MLQ_ERR_ARG, "mlq_set_attention_windows: layer %d window %d < 0", l, windows[l]);
            return MLQ_ERR_ARG;
        }
    }
    std::lock_guard<std::mutex> lk(g_win_mu);
    if (L == 0) g_windows.erase((uintptr_t)bc);
    else g_windows[(uintptr_t)bc] = std::vector<int>(windows, windows + L);
    return MLQ_OK;
}

void mlq_forget_model_plans(void) {
    destroy_graphs();
    std::lock_guard<std::mutex> lk(g_plan_mu);
    g_plans.clear();
}

int mlq_batch_forward(const void *bc, const int *tokens, int B, float *ws) {
    const BC *c = static_cast<const BC *>(bc);
    if (!c || !tokens || B <= 0 || B > 64 || c->L <= 0 || c->N <= 0 || c->NH <= 0 || c->NKH <= 0 ||
        c->NH % c->NKH || c->HD <= 0 || !c->kv_array || !c->logits || c->max_ctx <= 0 || c->N % 32) {
        set_error(MLQ_ERR_ARG, "batch_forward: bad model description or batch (B 1..64)");
        return MLQ_ERR_ARG;
    }
    const int L = c->L, N = c->N, NH = c->NH, NKH = c->NKH, HD = c->HD, inner = NH * HD, kvrow = NKH * HD;
    const int rope_dim = c->rope_dim > 0 ? c->rope_dim : HD;
    // Reference-compatibility mode reproduces the reference's data flow: every projection
    // reads the workspace's xn region (ws + B*S, never written by the reference), the
    // normalised activations overwrite x, and the fused QKV / QK projections hand
    // sequence b the Q slice at b*NH*HD of the projection buffer.
    const bool compat = ref_compat();
    int S = N;
    if (inner > S) S = inner;
    if (c->FF > S) S = c->FF;
    if (kvrow > S) S = kvrow;
    if (inner + kvrow > S) S = inner + kvrow;
    if (S < 8192) S = 8192;
    if (compat && !ws) {
        set_error(MLQ_ERR_ARG, "batch_forward: reference-compatibility mode reads the workspace; ws is NULL");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    Ctx *cx = ctx();
    if (!cx) return mlq_last_error();
    // ------------------------------------------------------------------ plan
    ModelPlan *P;
    {
        std::lock_guard<std::mutex> lk(g_plan_mu);
        auto key = std::make_pair(cx->device, (uintptr_t)c);
        auto fp = fingerprint(c);
        auto it = g_plans.find(key);
        if (it == g_plans.end() || it->second.fingerprint != fp) {
            ModelPlan np;
            if (!build_plan(c, cs, np)) return fwd_fail(cs, mlq_last_error() ? mlq_last_error() : MLQ_ERR_ARG);
            np.fingerprint = std::move(fp);
            static unsigned long long next_gen = 0;
            np.gen = ++next_gen;
            g_plans[key] = std::move(np);
            it = g_plans.find(key);
        }
        P = &it->second;
    }
    cudaStream_t s = stream();
    // ------------------------------------------------------------------ KV pages (host bookkeeping)
    std::vector<int> pos(B), tables((size_t)B * 1024);
    std::vector<float *> pools(B), mirror_k(B), mirror_v(B);
    int max_len = 0;
    MlqKVBlock *kv0 = c->kv_array[0];
    for (int b = 0; b < B; b++) {
        MlqKVBlock *kv = c->kv_array[b];
        if (!kv || !kv->pt.pages || !kv->pt.table || kv->pt._nkh != NKH || kv->pt._hd != HD || kv->pt._n_layers < L ||
            kv->pt.page_size != kv0->pt.page_size || kv->pt.n_pages != kv0->pt.n_pages ||
            kv->pt._n_layers != kv0->pt._n_layers || kv->pt.page_size <= 0 || kv->pt.n_pages <= 0) {
            set_error(MLQ_ERR_ARG, "batch_forward: KVBlock of sequence %d does not match the model", b);
            return fwd_fail(cs, MLQ_ERR_ARG);
        }
        if (!is_device_ptr(kv->pt.pages)) {
            set_error(MLQ_ERR_ARG, "batch_forward: KVBlock of sequence %d was not made by kv_init / page_table_init "
                                   "of this library (its pages are not device memory)", b);
            return fwd_fail(cs, MLQ_ERR_ARG);
        }
        const int p = kv->seq_len[0];
        const int blk = p / kv->pt.page_size;
        if (p >= c->max_ctx || blk >= 1024) {
            set_error(MLQ_ERR_CAPACITY, "batch_forward: sequence %d at position %d (max_ctx %d)", b, p, c->max_ctx);
            return fwd_fail(cs, MLQ_ERR_CAPACITY);
        }
        // every page below the new position must be mapped (attention reads them all)
        for (int i = 0; i < blk; i++) {
            if (kv->pt.table[i] < 0 || kv->pt.table[i] >= kv->pt.n_pages) {
                set_error(MLQ_ERR_ARG, "batch_forward: sequence %d has logical page %d unmapped (%d) below position %d",
                          b, i, kv->pt.table[i], p);
                return fwd_fail(cs, MLQ_ERR_ARG);
            }
        }
        if (kv->pt.table[blk] >= kv->pt.n_pages) {
            set_error(MLQ_ERR_ARG, "batch_forward: sequence %d maps page %d beyond the pool", b, kv->pt.table[blk]);
            return fwd_fail(cs, MLQ_ERR_ARG);
        }
        if (kv->pt.table[blk] < 0) {
            const int page = mlq_page_table_alloc(&kv->pt);
            if (page < 0) {
                set_error(MLQ_ERR_CAPACITY, "batch_forward: sequence %d: page pool full", b);
                return fwd_fail(cs, MLQ_ERR_CAPACITY);
            }
            kv->pt.table[blk] = page;
        }
        pos[b] = p;
        memcpy(&tables[(size_t)b * 1024], kv->pt.table, 1024 * sizeof(int));
        pools[b] = kv->pt.pages;
        // the KVBlock's own k/v arrays ([L][1024][64][row]) are written only when kv_init of
        // this library made them and the page geometry is the reference's (64 slots)
        const size_t need = (size_t)L * 1024 * 64 * kvrow * sizeof(float);
        const bool mirror = kv->pt.page_size == 64 && kv->k && kv->v && kv_array_bytes(kv->k) >= need &&
                            kv_array_bytes(kv->v) >= need;
        mirror_k[b] = mirror ? kv->k : nullptr;
        mirror_v[b] = mirror ? kv->v : nullptr;
        if (p + 1 > max_len) max_len = p + 1;
    }
    // ------------------------------------------------------------------ step
    std::vector<int> lens(B);
    for (int b = 0; b < B; b++) lens[b] = pos[b] + 1;
    bool any_ssm = false;
    for (int l = 0; l < L; l++) any_ssm |= P->layers[l].ssm;
    if (any_ssm && !c->ssm_state) {
        set_error(MLQ_ERR_ARG, "batch_forward: SSM layers without ssm_state");
        return fwd_fail(cs, MLQ_ERR_ARG);
    }
    StepDims d{B, N, inner, kvrow, c->FF, c->n_experts, c->n_experts_per_tok, c->moe_intermediate, c->outNR, NH, HD,
               L, any_ssm};
    d.gq = c->gate_exp_quant;
    d.uq = c->up_exp_quant;
    d.dq = c->down_exp_quant;
    const int tab_w = max_blocks_used(pos, kv0->pt.page_size);
    const float *ws_xn = compat ? ws + (size_t)B * S : nullptr;
    const bool graphable = graphs_enabled() && !(c->emb_quant == MLQ_Q4_K && !compat) && capturable(s);
    int rc;
    if (graphable) {
        rc = run_graph_step(c, P, d, compat, pos, lens, tables, pools, mirror_k, mirror_v, tab_w, max_len, tokens, ws_xn,
                            ws, s);
        if (rc == MLQ_OK) {
            for (int b = 0; b < B; b++) c->kv_array[b]->seq_len[0]++;
            cs.finish();
            return MLQ_OK;
        }
        if (rc != MLQ_ERR_UNSUPPORTED) return fwd_fail(cs, rc);
    }
    // direct launches with this call's scratch
    StepBufs sb;
    const size_t bytes = step_bytes(d);
    uint8_t *mem = (uint8_t *)cs.scratch(bytes);
    if (!mem) return fwd_fail(cs, mlq_last_error() ? mlq_last_error() : MLQ_ERR_CUDA);
    carve(sb, mem, d);
    const int *d_tok = (const int *)cs.in(tokens, sizeof(int) * B);
    const float *xin = compat ? (const float *)cs.in(ws_xn, sizeof(float) * (size_t)B * N) : nullptr;
    float *ws_out = ws ? (float *)cs.out(ws, sizeof(float) * (size_t)B * N) : nullptr;
    float *d_state = any_ssm ? (float *)cs.inout(c->ssm_state, sizeof(float) * (size_t)L * kSsmGroups * kSsmState)
                             : nullptr;
    float *d_logits = (float *)cs.out(c->logits, sizeof(float) * (size_t)B * c->outNR);
    if (cs.failed) return cs.finish();
    rc = upload_step_inputs(sb, d, pos, lens, tables, pools, mirror_k, mirror_v, tab_w, s);
    if (rc == MLQ_OK) {
        std::vector<int> th(B, 0);   // host ids are needed only by the per-row Q4_K decode
        if (c->emb_quant == MLQ_Q4_K && !compat && !host_tokens(tokens, B, th)) rc = MLQ_ERR_CUDA;
        if (rc == MLQ_OK)
            rc = enqueue_step(c, P, sb, d, compat, max_len, tab_w, d_tok, th.data(), xin, d_state,
                              ws_out ? ws_out : sb.xn, d_logits, s);
    }
    if (rc != MLQ_OK) return fwd_fail(cs, rc);
    for (int b = 0; b < B; b++) c->kv_array[b]->seq_len[0]++;
    return cs.finish();
}

// moe_ffn (cengine_batch_instr.c:591-665): for each of the B tokens of x [B][N], F32 router
// of layer l, softmax, top-k without renormalisation, experts, weighted sum -> ffn [B][N]
// (the reference keeps only the last token's result in its single ffn_buf; every token's
// row is written here).
int mlq_moe_ffn(const void *bc, int l, const float *x, float *ffn, int B) {
    const BC *c = static_cast<const BC *>(bc);
    if (!c || !x || !ffn || B <= 0 || l < 0 || l >= c->L || c->n_experts <= 0 || c->n_experts_per_tok <= 0 ||
        !c->w_gate_inp || !c->w_gate_exps || !c->w_up_exps || !c->w_down_exps) {
        set_error(MLQ_ERR_ARG, "moe_ffn: bad arguments or no MoE in the model");
        return MLQ_ERR_ARG;
    }
    const int N = c->N, E = c->n_experts, k = c->n_experts_per_tok, M = c->moe_intermediate;
    const long long gs = expert_stride(c->gate_exp_quant, M, N, false);
    const long long us = expert_stride(c->up_exp_quant, M, N, false);
    const long long ds = expert_stride(c->down_exp_quant, N, M, true);
    if (!gs || !us || !ds) { set_error(MLQ_ERR_TYPE, "moe_ffn: expert types"); return MLQ_ERR_TYPE; }
    CallScope cs;
    const float *router = (const float *)cs.weights(c->w_gate_inp[l], sizeof(float) * (size_t)E * N);
    const uint8_t *gexp = (const uint8_t *)cs.weights(c->w_gate_exps[l], expert_extent(gs, E, c->gate_exp_quant, M, N));
    const uint8_t *uexp = (const uint8_t *)cs.weights(c->w_up_exps[l], expert_extent(us, E, c->up_exp_quant, M, N));
    const uint8_t *dexp = (const uint8_t *)cs.weights(c->w_down_exps[l], expert_extent(ds, E, c->down_exp_quant, N, M));
    const float *dx = (const float *)cs.in(x, sizeof(float) * (size_t)B * N);
    float *logits = (float *)cs.scratch(sizeof(float) * (size_t)B * E);
    int *idx = (int *)cs.scratch(sizeof(int) * (size_t)B * k);
    float *w = (float *)cs.scratch(sizeof(float) * (size_t)B * k);
    float *hm = (float *)cs.scratch(sizeof(float) * (size_t)B * k * M);
    float *hm2 = (float *)cs.scratch(sizeof(float) * (size_t)B * k * M);
    float *dout = (float *)cs.out(ffn, sizeof(float) * (size_t)B * N);
    if (cs.failed) return cs.finish();
    cudaStream_t s = stream();
    int rc = launch_matmul((const uint8_t *)router, MLQ_F32, dx, logits, E, N, B, 0, s);
    if (rc == MLQ_OK) rc = launch_router_topk(logits, B, E, k, 0, idx, w, s);
    if (rc == MLQ_OK)
        rc = launch_moe_experts(c->gate_exp_quant, c->up_exp_quant, c->down_exp_quant, gexp, uexp, dexp, gs, us, ds,
                                idx, w, k, B, M, N, dx, hm, hm2, dout, nullptr, HUGE_VALF, s);
    if (rc != MLQ_OK) return fwd_fail(cs, rc);
    return cs.finish();
}

}  // extern "C"
