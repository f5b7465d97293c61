// Mixture-of-experts FFN of the reference engine on the GPU.
//
// Replaces moe_forward_omp (quant_kernels_omp.c:2066-2250), the routers of
// moe_ffn / qwen36_batch_forward / router_topk (cengine_batch_instr.c:615-646,
// 1113-1152; gptoss_batch_forward.c:53-93) and the per-expert loop of moe_ffn.
//
// k_moe_gemv: a grouped GEMV whose tile is the same `rpt` rows of G matrices (the
// selected experts' gate/up, or their down projections).  The producer warp streams
// the G row-ranges of a tile into one shared-memory stage (one cp.async.bulk each);
// the 8 decode warps compute the G*rpt row dots (weights decoded from the staged
// GGUF blocks, activations from int8 planes, dp4a) and an epilogue combines them:
//   MOE_SWIGLU  matrices come as (gate_e, up_e) pairs:
//               h_e[r] = silu(clamp(gate, -80, 80)) * up      (quant_kernels_omp.c:2157-2164)
//   MOE_WSUM    out[r] = sum_g w_g * dot_g(r) (+ residual[r]), g in order -- the
//               weighted combine of the down projections, deterministic (the
//               reference accumulates with `omp atomic`, :2199-2243)
//   MOE_STORE   out[g][r] = dot_g(r)
// A token's MoE layer is therefore two launches: gate/up/SwiGLU, then down/combine.
// Roofline: HBM-bound on the selected experts' weight bytes (k * 3 matrices).
#include <cuda_runtime.h>
#include <math.h>
#include <stdlib.h>

#include <map>
#include <vector>

#include "formats.cuh"
#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

constexpr int kMoeMaxG = 32;
constexpr int kMoeWarps = 8;
constexpr int kMoeThreads = (kMoeWarps + 1) * 32;
constexpr int kMoeMaxStages = 6;
constexpr int kMoeSmemBudget = 200 * 1024;
enum { MOE_SWIGLU = 0, MOE_WSUM = 1, MOE_STORE = 2 };

struct MoeArgs {
    const uint8_t *W[kMoeMaxG];
    float wgt[kMoeMaxG];
    int G, n_rows, K;
    long long row_bytes;
    int rpt, n_tiles, slot_bytes, n_stages;
    const float *x;      // [nx][K]; matrix g uses activation row (nx == 1 ? 0 : g)
    int nx;
    float *out;
    const float *residual;
    int *status;
    // indexed mode (routing stays on the device): matrix g is expert e = idx[g / per] of
    // the expert tensor base[g % per] (stride estride bytes per expert), weight w[g];
    // per = 2 for SwiGLU (gate, up), 1 otherwise.  Token t = blockIdx.y reads idx/w at
    // t * G / per, x at t * x_tok, writes out at t * out_tok, residual at t * out_tok.
    int indexed;
    const int *idx;
    const float *w;
    const uint8_t *base[2];
    long long estride;
    long long x_tok, out_tok;
    float clamp;   // SwiGLU gate clamp (+-80 for moe_forward_omp; infinity for moe_ffn)
};

__device__ __forceinline__ const uint8_t *moe_mat(const MoeArgs &a, int g) {
    if (!a.indexed) return a.W[g];
    const int per = (a.G > 0 && a.base[1]) ? 2 : 1;
    const int e = a.idx[(size_t)blockIdx.y * (a.G / per) + g / per];
    if (e < 0) return nullptr;
    return a.base[g % per] + (size_t)e * a.estride;
}

__device__ __forceinline__ float moe_wgt(const MoeArgs &a, int g) {
    return a.indexed ? a.w[(size_t)blockIdx.y * a.G + g] : a.wgt[g];
}

struct MoeLayout {
    int off_bar, off_flag, off_xh, off_xl, off_xs, off_xsum, off_res, off_stage, total;
};

__host__ __device__ inline int mo_align(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ inline MoeLayout moe_layout(int nx, int K, int G, int rpt, int slot_bytes, int n_stages) {
    MoeLayout L;
    int o = 0;
    L.off_bar = o;  o += 2 * kMoeMaxStages * 8;
    L.off_flag = o; o += 16;
    o = mo_align(o, 128);
    L.off_xh = o;   o = mo_align(o + nx * K, 16);
    L.off_xl = o;   o = mo_align(o + nx * K, 16);
    L.off_xs = o;   o += nx * (K / 32) * 4;
    L.off_xsum = o; o = mo_align(o + nx * (K / 32) * 4, 16);
    L.off_res = o;  o = mo_align(o + 2 * G * rpt * 4, 128);
    L.off_stage = o; o += n_stages * G * slot_bytes;
    L.total = o;
    return L;
}

template <int QT, int MODE>
__global__ void __launch_bounds__(kMoeThreads, 1) k_moe_gemv(MoeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const MoeLayout L = moe_layout(a.nx, a.K, a.G, a.rpt, a.slot_bytes, a.n_stages);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.off_bar);
    uint64_t *empty = full + kMoeMaxStages;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.off_flag);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_iter = (a.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
    const long long tile_bytes = (long long)a.rpt * a.row_bytes;
    const long long total = (long long)a.n_rows * a.row_bytes;
    const int stage_bytes = a.G * a.slot_bytes;
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.n_stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMoeWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kMoeWarps) {
        // ---------------------------------------------------------------- producer
        const uint64_t pol = policy_evict_first();
        for (int it = 0; it < n_iter; ++it) {
            const int s = it % a.n_stages;
            if (it >= a.n_stages) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait_bounded(&empty[s], ((it / a.n_stages) - 1) & 1);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok || *abort_flag) {
                    if (lane == 0) { *abort_flag = 1; report_status(a.status, DEV_ST_WAIT_EMPTY); }
                    return;
                }
            }
            const long long tile = (long long)blockIdx.x + (long long)it * gridDim.x;
            const long long b0 = tile * tile_bytes, b1 = min(b0 + tile_bytes, total);
            uint32_t tx = 0;
            for (int g = 0; g < a.G; g++) {
                const uint8_t *Wg = moe_mat(a, g);
                if (!Wg) continue;
                const uintptr_t g0 = reinterpret_cast<uintptr_t>(Wg) + (uintptr_t)b0;
                const uintptr_t g1 = reinterpret_cast<uintptr_t>(Wg) + (uintptr_t)b1;
                const uintptr_t gd = g0 & ~uintptr_t(15);
                const uintptr_t i0 = (g0 + 15) & ~uintptr_t(15), i1 = g1 & ~uintptr_t(15);
                uint8_t *st = smem + L.off_stage + (size_t)s * stage_bytes + (size_t)g * a.slot_bytes;
                if (i1 > i0) {
                    if (g0 + lane < i0) st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
                    if (i1 + lane < g1) st[i1 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(i1 + lane));
                    tx += (uint32_t)(i1 - i0);
                } else if (g0 + lane < g1) {
                    st[g0 + lane - gd] = ldg_u8_nc(reinterpret_cast<const uint8_t *>(g0 + lane));
                }
            }
            __syncwarp();
            if (lane == 0) {
                if (tx) {
                    mbar_arrive_expect_tx(&full[s], tx);
                    for (int g = 0; g < a.G; g++) {
                        const uint8_t *Wg = moe_mat(a, g);
                        if (!Wg) continue;
                        const uintptr_t g0 = reinterpret_cast<uintptr_t>(Wg) + (uintptr_t)b0;
                        const uintptr_t g1 = reinterpret_cast<uintptr_t>(Wg) + (uintptr_t)b1;
                        const uintptr_t gd = g0 & ~uintptr_t(15);
                        const uintptr_t i0 = (g0 + 15) & ~uintptr_t(15), i1 = g1 & ~uintptr_t(15);
                        if (i1 > i0) {
                            uint8_t *st = smem + L.off_stage + (size_t)s * stage_bytes + (size_t)g * a.slot_bytes;
                            bulk_g2s(st + (i0 - gd), reinterpret_cast<const void *>(i0), (uint32_t)(i1 - i0), &full[s], pol);
                        }
                    }
                } else {
                    mbar_arrive(&full[s]);
                }
            }
        }
        return;
    }

    // -------------------------------------------------------------------- decode warps
    int8_t *xh = reinterpret_cast<int8_t *>(smem + L.off_xh);
    int8_t *xl = reinterpret_cast<int8_t *>(smem + L.off_xl);
    float *xs = reinterpret_cast<float *>(smem + L.off_xs);
    float *xsum = reinterpret_cast<float *>(smem + L.off_xsum);
    float *res = reinterpret_cast<float *>(smem + L.off_res);
    const float *xt = a.x + (size_t)blockIdx.y * a.x_tok;
    for (int m = 0; m < a.nx; m++)
        encode_x_planes<1>(xt + (size_t)m * a.K, 1, a.K, xh + (size_t)m * a.K, xl + (size_t)m * a.K,
                           xs + (size_t)m * (a.K / 32), xsum + (size_t)m * (a.K / 32), warp, lane, kMoeWarps);
    float *out = a.out + (size_t)blockIdx.y * a.out_tok;
    const float *residual = a.residual ? a.residual + (size_t)blockIdx.y * a.out_tok : nullptr;
    named_bar_sync(1, kMoeWarps * 32);
    const int U = a.K / Fmt<QT>::UE;
    const int items = a.G * a.rpt;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % a.n_stages;
        bool ok = false;
        if (!*abort_flag) {
            if (lane == 0) ok = mbar_wait_bounded(&full[s], (it / a.n_stages) & 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok && lane == 0) { *abort_flag = 1; report_status(a.status, DEV_ST_WAIT_FULL); }
        }
        const long long tile = (long long)blockIdx.x + (long long)it * gridDim.x;
        const int row0 = (int)(tile * a.rpt);
        float *rs = res + (it & 1) * items;
        for (int i = warp; i < items; i += kMoeWarps) {
            const int g = i / a.rpt, r = i - g * a.rpt;
            float acc[1] = {0.0f};
            const uint8_t *Wg = moe_mat(a, g);
            if (ok && Wg && row0 + r < a.n_rows) {
                const int xr = (a.nx == 1) ? 0 : g;
                const XPlanes xp{xh + (size_t)xr * a.K, xl + (size_t)xr * a.K, xs + (size_t)xr * (a.K / 32),
                                 xsum + (size_t)xr * (a.K / 32), a.K, a.K, a.K / 32};
                const uintptr_t g0 = reinterpret_cast<uintptr_t>(Wg) + (uintptr_t)(tile * tile_bytes);
                const uint8_t *rowp = smem + L.off_stage + (size_t)s * stage_bytes + (size_t)g * a.slot_bytes +
                                      (g0 & 15) + (size_t)r * a.row_bytes;
                for (int u = lane; u < U; u += 32) Unit<QT, 1>::dot(rowp, u, xp, acc);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
            if (lane == 0) rs[i] = acc[0];
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&empty[s]);
        named_bar_sync(1, kMoeWarps * 32);
        if (!ok) continue;
        if (MODE == MOE_SWIGLU) {
            const int pairs = a.G / 2;
            for (int t = threadIdx.x; t < pairs * a.rpt; t += kMoeWarps * 32) {
                const int e = t / a.rpt, r = t - e * a.rpt;
                if (row0 + r < a.n_rows) {
                    float gv = fminf(fmaxf(rs[(2 * e) * a.rpt + r], -a.clamp), a.clamp);
                    out[(size_t)e * a.n_rows + row0 + r] = (gv / (1.0f + expf(-gv))) * rs[(2 * e + 1) * a.rpt + r];
                }
            }
        } else if (MODE == MOE_WSUM) {
            for (int r = threadIdx.x; r < a.rpt; r += kMoeWarps * 32) {
                if (row0 + r < a.n_rows) {
                    float sum = residual ? residual[row0 + r] : 0.0f;
                    for (int g = 0; g < a.G; g++) sum = fmaf(moe_wgt(a, g), rs[g * a.rpt + r], sum);
                    out[row0 + r] = sum;
                }
            }
        } else {
            for (int t = threadIdx.x; t < items; t += kMoeWarps * 32) {
                const int g = t / a.rpt, r = t - g * a.rpt;
                if (row0 + r < a.n_rows) out[(size_t)g * a.n_rows + row0 + r] = rs[t];
            }
        }
    }
}

template <int QT, int MODE>
static int launch_moe_t(MoeArgs &a, int n_tok, cudaStream_t s) {
    const LaunchEnv *env = launch_env();
    if (!env) return MLQ_ERR_NO_DEVICE;
    const long long rb = a.row_bytes;
    int rpt = (int)(32768 / (a.G * rb));
    rpt = rpt < 1 ? 1 : (rpt > 16 ? 16 : rpt);
    while (rpt > 1 && (a.n_rows + rpt - 1) / rpt < env->num_sms) rpt >>= 1;
    a.rpt = rpt;
    a.slot_bytes = mo_align((int)(rpt * rb), 16) + 48;
    const int fixed = moe_layout(a.nx, a.K, a.G, rpt, a.slot_bytes, 0).total;
    int n_stages = (kMoeSmemBudget - fixed) / (a.G * a.slot_bytes);
    if (n_stages > kMoeMaxStages) n_stages = kMoeMaxStages;
    if (n_stages < 2) {
        set_error(MLQ_ERR_CAPACITY, "moe: %d matrices x K=%d do not fit the shared-memory ring", a.G, a.K);
        return MLQ_ERR_CAPACITY;
    }
    a.n_stages = n_stages;
    a.n_tiles = (a.n_rows + rpt - 1) / rpt;
    a.status = env->d_status;
    const int smem = fixed + n_stages * a.G * a.slot_bytes;
    static bool attr = false;
    if (!attr) {
        if (!MLQ_CUDA(cudaFuncSetAttribute(k_moe_gemv<QT, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448)))
            return MLQ_ERR_CUDA;
        attr = true;
    }
    int gx = a.n_tiles < env->num_sms ? a.n_tiles : env->num_sms;
    if (n_tok > 1) {
        gx = (env->num_sms + n_tok - 1) / n_tok;
        if (gx > a.n_tiles) gx = a.n_tiles;
        if (gx < 1) gx = 1;
    }
    k_moe_gemv<QT, MODE><<<dim3(gx, n_tok), kMoeThreads, smem, s>>>(a);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

template <int MODE>
static int launch_moe_mode(int qt, MoeArgs &a, int n_tok, cudaStream_t s) {
    switch (qt) {
        case MLQ_Q4_0: return launch_moe_t<MLQ_Q4_0, MODE>(a, n_tok, s);
        case MLQ_Q4_1: return launch_moe_t<MLQ_Q4_1, MODE>(a, n_tok, s);
        case MLQ_Q5_0: return launch_moe_t<MLQ_Q5_0, MODE>(a, n_tok, s);
        case MLQ_Q8_0: return launch_moe_t<MLQ_Q8_0, MODE>(a, n_tok, s);
        case MLQ_Q4_K: return launch_moe_t<MLQ_Q4_K, MODE>(a, n_tok, s);
        case MLQ_Q5_K: return launch_moe_t<MLQ_Q5_K, MODE>(a, n_tok, s);
        case MLQ_Q6_K: return launch_moe_t<MLQ_Q6_K, MODE>(a, n_tok, s);
        case MLQ_MXFP4: return launch_moe_t<MLQ_MXFP4, MODE>(a, n_tok, s);
        case MLQ_MXFP4_REF: return launch_moe_t<MLQ_MXFP4_REF, MODE>(a, n_tok, s);
        default:
            set_error(MLQ_ERR_TYPE, "moe: expert type %d not supported on the grouped path", qt);
            return MLQ_ERR_TYPE;
    }
}

// G matrices W[g] (n_rows x K, type qt) against activations x [nx][K]
int launch_moe_gemv(int mode, int qt, const uint8_t *const *W, const float *wgt, int G, int n_rows, int K,
                    const float *x, int nx, float *out, const float *residual, cudaStream_t s) {
    if (G < 1 || G > kMoeMaxG || (mode == MOE_SWIGLU && G % 2)) {
        set_error(MLQ_ERR_ARG, "moe: %d matrices per launch (1..%d, even for SwiGLU)", G, kMoeMaxG);
        return MLQ_ERR_ARG;
    }
    if (ref_compat() && qt == MLQ_MXFP4) qt = MLQ_MXFP4_REF;
    MoeArgs a{};
    a.clamp = 80.0f;
    for (int g = 0; g < G; g++) {
        a.W[g] = W[g];
        a.wgt[g] = wgt ? wgt[g] : 0.0f;
    }
    a.G = G;
    a.n_rows = n_rows;
    a.K = K;
    a.row_bytes = (long long)(K / block_elems(qt)) * block_bytes(qt);
    a.x = x;
    a.nx = nx;
    a.out = out;
    a.residual = residual;
    if (mode == MOE_SWIGLU) return launch_moe_mode<MOE_SWIGLU>(qt, a, 1, s);
    if (mode == MOE_WSUM) return launch_moe_mode<MOE_WSUM>(qt, a, 1, s);
    return launch_moe_mode<MOE_STORE>(qt, a, 1, s);
}

// Routing on the device: n_tok tokens, top_k experts each from d_idx / d_w [n_tok][top_k].
// SwiGLU: experts' gate (base_a) and up (base_b) n_ff x K, x [n_tok][K] -> h [n_tok][top_k][n_ff].
// Store: experts' matrices (base_a) n_rows x K, x [n_tok][K] -> out [n_tok][top_k][n_rows].
// Weighted sum: experts' down (base_a) N x n_ff, h [n_tok][top_k][n_ff] -> out [n_tok][N]
// (+ residual [n_tok][N]).
int launch_moe_indexed(int mode, int qt, const uint8_t *base_a, const uint8_t *base_b, long long expert_stride,
                       const int *d_idx, const float *d_w, int top_k, int n_tok, int n_rows, int K, const float *x,
                       float *out, const float *residual, cudaStream_t s, float swiglu_clamp) {
    const int G = (mode == MOE_SWIGLU) ? 2 * top_k : top_k;
    if (G < 1 || G > kMoeMaxG || n_tok < 1 || n_tok > 65535) {
        set_error(MLQ_ERR_ARG, "moe: top_k %d / tokens %d out of range", top_k, n_tok);
        return MLQ_ERR_ARG;
    }
    if (ref_compat() && qt == MLQ_MXFP4) qt = MLQ_MXFP4_REF;
    MoeArgs a{};
    a.G = G;
    a.n_rows = n_rows;
    a.K = K;
    a.row_bytes = (long long)(K / block_elems(qt)) * block_bytes(qt);
    a.indexed = 1;
    a.clamp = swiglu_clamp;
    a.idx = d_idx;
    a.w = d_w;
    a.base[0] = base_a;
    a.base[1] = (mode == MOE_SWIGLU) ? base_b : nullptr;
    a.estride = expert_stride;
    a.x = x;
    a.residual = residual;
    a.out = out;
    if (mode == MOE_SWIGLU || mode == MOE_STORE) {
        a.nx = 1;
        a.x_tok = K;
        a.out_tok = (long long)top_k * n_rows;
        return mode == MOE_SWIGLU ? launch_moe_mode<MOE_SWIGLU>(qt, a, n_tok, s)
                                  : launch_moe_mode<MOE_STORE>(qt, a, n_tok, s);
    }
    a.nx = top_k;
    a.x_tok = (long long)top_k * K;
    a.out_tok = n_rows;
    return launch_moe_mode<MOE_WSUM>(qt, a, n_tok, s);
}

__global__ void k_swiglu_clamp(float *__restrict__ h, const float *__restrict__ g, const float *__restrict__ u,
                               long long n, float clamp) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float gv = fminf(fmaxf(g[i], -clamp), clamp);
        h[i] = (gv / (1.0f + expf(-gv))) * u[i];
    }
}

// Routed experts of n_tok tokens with the routing on the device:
//   h_t,i = silu(clamp(gate_e x_t)) * (up_e x_t)  for e = idx[t][i], i < top_k
//   out_t = residual_t + sum_i w[t][i] * down_e h_t,i       (fixed order i = 0..top_k-1)
// Gate and up of one type and stride share one launch (fused SwiGLU epilogue); otherwise
// each is stored ([n_tok][top_k][n_ff] in h and h2) and combined elementwise.  out may
// alias residual.
int launch_moe_experts(int gqt, int uqt, int dqt, const uint8_t *gexp, const uint8_t *uexp, const uint8_t *dexp,
                       long long gs, long long us, long long ds, const int *idx, const float *w, int top_k,
                       int n_tok, int n_ff, int N, const float *x, float *h, float *h2, float *out,
                       const float *residual, float clamp, cudaStream_t s) {
    int rc;
    if (gqt == uqt && gs == us) {
        rc = launch_moe_indexed(MOE_SWIGLU, gqt, gexp, uexp, gs, idx, w, top_k, n_tok, n_ff, N, x, h, nullptr, s,
                                clamp);
    } else {
        rc = launch_moe_indexed(MOE_STORE, gqt, gexp, nullptr, gs, idx, w, top_k, n_tok, n_ff, N, x, h, nullptr, s);
        if (rc == MLQ_OK)
            rc = launch_moe_indexed(MOE_STORE, uqt, uexp, nullptr, us, idx, w, top_k, n_tok, n_ff, N, x, h2, nullptr,
                                    s);
        if (rc == MLQ_OK) {
            const long long n = (long long)n_tok * top_k * n_ff;
            long long g = (n + 255) / 256;
            k_swiglu_clamp<<<(int)(g > 4096 ? 4096 : g), 256, 0, s>>>(h, h, h2, n, clamp);
            count_launch();
            rc = MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
        }
    }
    if (rc != MLQ_OK) return rc;
    return launch_moe_indexed(MOE_WSUM, dqt, dexp, nullptr, ds, idx, w, top_k, n_tok, N, n_ff, h, out, residual, s);
}

// ------------------------------------------------------------------------------ router
// One warp per token: softmax over E logits (1/(sum + 1e-10)), top-k by the reference's
// insertion rule (strictly greater wins, so ties keep the lower expert index), optional
// renormalisation of the k weights (1/(sum + 1e-10)).
__global__ void k_router_topk(const float *__restrict__ logits, int B, int E, int k, int renorm,
                              int *__restrict__ idx, float *__restrict__ w) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int b = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (b >= B) return;
    const float *lg = logits + (size_t)b * E;
    // lane holds experts lane + 32 j (j < 8: up to 256 experts) in registers
    float p[8];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int e = lane + 32 * j;
        p[j] = e < E ? lg[e] : -INFINITY;
        mx = fmaxf(mx, p[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        p[j] = (lane + 32 * j) < E ? expf(p[j] - mx) : 0.0f;
        sum += p[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / (sum + 1e-10f);
#pragma unroll
    for (int j = 0; j < 8; j++) p[j] = (lane + 32 * j) < E ? p[j] * inv : -INFINITY;
    float tsum = 0.0f;
    for (int s = 0; s < k; s++) {
        // this lane's best remaining expert (strictly greater wins: ties keep the lower index)
        float best = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (p[j] > best) { best = p[j]; bi = lane + 32 * j; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (bi >= 0 && bi < E && (bi & 31) == lane) {
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (lane + 32 * j == bi) p[j] = -INFINITY;   // taken
        }
        if (lane == 0) {
            idx[(size_t)b * k + s] = (bi < E) ? bi : -1;
            w[(size_t)b * k + s] = best;
        }
        tsum += best;
    }
    if (renorm && lane == 0) {
        const float ti = 1.0f / (tsum + 1e-10f);
        for (int s = 0; s < k; s++) w[(size_t)b * k + s] *= ti;
    }
}

int launch_router_topk(const float *logits, int B, int E, int k, int renorm, int *idx, float *w, cudaStream_t s) {
    if (E > 256 || k < 1 || k > E) {
        set_error(MLQ_ERR_CAPACITY, "router: %d experts, top-%d (at most 256 experts)", E, k);
        return MLQ_ERR_CAPACITY;
    }
    return MLQ_CUDA(launch_pdl_k(k_router_topk, dim3((B * 32 + 127) / 128), dim3(128), 0, s, logits, B, E, k, renorm, idx, w)) ? MLQ_OK : MLQ_ERR_CUDA;
}

}  // namespace mlq

// ====================================================================================== C-ABI
using namespace mlq;

extern "C" {

// moe_forward_omp semantics with GGUF-correct math for every expert type:
// combined = sum_i w[i] * W_down[idx[i]] . (silu(clamp(W_gate[idx[i]] x)) * (W_up[idx[i]] x))
int mlq_moe_forward(const void *const *gate, const void *const *up, const void *const *down, const float *x,
                    int n_ff, int n_embd, int qt_gate, int qt_up, int qt_down, const int *top_idx,
                    const float *top_w, int top_k, float *combined) {
    if (!gate || !up || !down || !x || !top_idx || !top_w || !combined || n_ff <= 0 || n_embd <= 0 ||
        top_k <= 0 || 2 * top_k > kMoeMaxG) {
        set_error(MLQ_ERR_ARG, "mlq_moe_forward: bad arguments (top_k 1..%d)", kMoeMaxG / 2);
        return MLQ_ERR_ARG;
    }
    const size_t rb_g = mlq_row_bytes(qt_gate, n_embd), rb_u = mlq_row_bytes(qt_up, n_embd);
    const size_t rb_d = mlq_row_bytes(qt_down, n_ff);
    if (!rb_g || !rb_u || !rb_d) {
        set_error(MLQ_ERR_TYPE, "mlq_moe_forward: types %d/%d/%d with n_embd %d, n_ff %d", qt_gate, qt_up, qt_down,
                  n_embd, n_ff);
        return MLQ_ERR_TYPE;
    }
    // the selected experts and their weights are read on the host (as the reference does)
    std::vector<int> idx(top_k);
    std::vector<float> w(top_k);
    const bool idx_dev = is_device_ptr(top_idx), w_dev = is_device_ptr(top_w);
    if (idx_dev) cudaMemcpy(idx.data(), top_idx, sizeof(int) * top_k, cudaMemcpyDeviceToHost);
    else for (int i = 0; i < top_k; i++) idx[i] = top_idx[i];
    if (w_dev) cudaMemcpy(w.data(), top_w, sizeof(float) * top_k, cudaMemcpyDeviceToHost);
    else for (int i = 0; i < top_k; i++) w[i] = top_w[i];
    CallScope cs;
    std::vector<const uint8_t *> gu(2 * top_k), dn(top_k);
    for (int i = 0; i < top_k; i++) {
        if (idx[i] < 0) {
            set_error(MLQ_ERR_ARG, "mlq_moe_forward: expert index %d", idx[i]);
            return MLQ_ERR_ARG;
        }
        gu[2 * i] = (const uint8_t *)cs.weights(gate[idx[i]], rb_g * n_ff);
        gu[2 * i + 1] = (const uint8_t *)cs.weights(up[idx[i]], rb_u * n_ff);
        dn[i] = (const uint8_t *)cs.weights(down[idx[i]], rb_d * n_embd);
    }
    const float *dx = (const float *)cs.in(x, sizeof(float) * (size_t)n_embd);
    float *h = (float *)cs.scratch(sizeof(float) * (size_t)top_k * n_ff);
    float *dout = (float *)cs.out(combined, sizeof(float) * (size_t)n_embd);
    if (cs.failed) return cs.finish();
    cudaStream_t s = stream();
    int rc;
    if (qt_gate == qt_up) {
        rc = launch_moe_gemv(MOE_SWIGLU, qt_gate, gu.data(), nullptr, 2 * top_k, n_ff, n_embd, dx, 1, h, nullptr, s);
    } else {
        float *gbuf = (float *)cs.scratch(sizeof(float) * (size_t)2 * top_k * n_ff);
        std::vector<const uint8_t *> gs(top_k), us(top_k);
        for (int i = 0; i < top_k; i++) { gs[i] = gu[2 * i]; us[i] = gu[2 * i + 1]; }
        rc = launch_moe_gemv(MOE_STORE, qt_gate, gs.data(), nullptr, top_k, n_ff, n_embd, dx, 1, gbuf, nullptr, s);
        if (rc == MLQ_OK)
            rc = launch_moe_gemv(MOE_STORE, qt_up, us.data(), nullptr, top_k, n_ff, n_embd, dx, 1,
                                 gbuf + (size_t)top_k * n_ff, nullptr, s);
        if (rc == MLQ_OK) rc = launch_swiglu(h, gbuf, gbuf + (size_t)top_k * n_ff, (long long)top_k * n_ff, s);
    }
    if (rc == MLQ_OK)
        rc = launch_moe_gemv(MOE_WSUM, qt_down, dn.data(), w.data(), top_k, n_embd, n_ff, h, top_k, dout, nullptr, s);
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

// logits = W_r x (W_r: E x N of type qt_r), softmax, top-k, optional renormalisation.
// x [B][N] -> idx [B][k], w [B][k]
int mlq_moe_router(const float *x, int B, int N, const void *W_r, int qt_r, int E, int k, int renorm, int *idx,
                   float *w) {
    if (!x || !W_r || !idx || !w || B <= 0 || N <= 0 || E <= 0 || k <= 0 || k > E) {
        set_error(MLQ_ERR_ARG, "mlq_moe_router: bad arguments");
        return MLQ_ERR_ARG;
    }
    const size_t rb = mlq_row_bytes(qt_r, N);
    if (!rb) { set_error(MLQ_ERR_TYPE, "mlq_moe_router: type %d, N %d", qt_r, N); return MLQ_ERR_TYPE; }
    CallScope cs;
    const uint8_t *dW = (const uint8_t *)cs.weights(W_r, rb * E);
    const float *dx = (const float *)cs.in(x, sizeof(float) * (size_t)B * N);
    float *logits = (float *)cs.scratch(sizeof(float) * (size_t)B * E);
    int *di = (int *)cs.out(idx, sizeof(int) * (size_t)B * k);
    float *dw = (float *)cs.out(w, sizeof(float) * (size_t)B * k);
    if (cs.failed) return cs.finish();
    int rc = launch_matmul(dW, qt_r, dx, logits, E, N, B, rb * E, stream());
    if (rc == MLQ_OK) rc = launch_router_topk(logits, B, E, k, renorm, di, dw, stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

}  // extern "C"
