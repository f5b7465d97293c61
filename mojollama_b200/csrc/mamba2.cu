// Mamba-2 decode step: the selective state-space update of one token per sequence.
//
// The reference has no real Mamba-2 (its ssm_decode_step, cengine_batch_instr.c:736-797, is
// a toy kept byte-compatible in ssm.cu).  This is the published recurrence (Dao & Gu,
// "Transformers are SSMs", 2024) under its own names, mlq_mamba2_step / mlq_mamba2_layer,
// for config 5's hybrid model (16 heads x 128, state 128, conv width 4):
//   conv:  window = last d_conv inputs of xBC (newest last); a = silu(bias + w . window)
//   a -> x [H][P] | B [G][S] | C [G][S]; head h reads group h / (H / G)
//   dt_h = softplus(dt_h + dt_bias_h) (clamped at 0); A_h = -exp(A_log_h)
//   state[h] = exp(dt_h A_h) state[h] + dt_h x[h] B^T;   y[h] = state[h] C + D_h x[h]
//   y = norm_w * rmsnorm(y * silu(z)) over groups of norm_group elements (optional)
// Three launches, each waiting on its predecessor with programmatic dependent launch:
//   k_m2_conv   one thread per (sequence, channel): roll the window, write the activation
//   k_m2_scan   one CTA per (sequence, head, 32 state rows): the state rows stream through
//               registers once (read + write), B and C of the head's group in shared memory
//   k_m2_norm   one CTA per (sequence, norm group), only with norm_w
// Roofline: HBM-bound on the SSM state, 2 * B * H * P * S * 4 bytes per step (config 5,
// B = 10: 21 MB).  Shapes: conv_state [B][conv_dim][d_conv], ssm_state [B][H][P][S].
#include <cuda_runtime.h>
#include <math.h>

#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

constexpr int kM2MaxConv = 8;
constexpr int kM2Rows = 32;        // state rows per scan CTA
constexpr int kM2Threads = 256;

__device__ __forceinline__ float m2_silu(float v) { return v / (1.0f + __expf(-v)); }

__device__ __forceinline__ float m2_softplus(float v) { return v > 20.0f ? v : log1pf(__expf(v)); }

__global__ void __launch_bounds__(256) k_m2_conv(const float *__restrict__ xbc, int xbc_stride,
                                                 float *__restrict__ conv_state, const float *__restrict__ conv_w,
                                                 const float *__restrict__ conv_b, float *__restrict__ act,
                                                 int conv_dim, int K) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= conv_dim) return;
    float *st = conv_state + ((size_t)b * conv_dim + c) * K;
    const float *w = conv_w + (size_t)c * K;
    float win[kM2MaxConv];
    if (K == 4) {
        const float4 s4 = *reinterpret_cast<const float4 *>(st);
        win[0] = s4.y; win[1] = s4.z; win[2] = s4.w;
    } else {
        for (int k = 0; k + 1 < K; k++) win[k] = st[k + 1];
    }
    win[K - 1] = xbc[(size_t)b * xbc_stride + c];
    float acc = conv_b ? conv_b[c] : 0.0f;
    for (int k = 0; k < K; k++) acc = fmaf(w[k], win[k], acc);
    if (K == 4) {
        *reinterpret_cast<float4 *>(st) = make_float4(win[0], win[1], win[2], win[3]);
    } else {
        for (int k = 0; k < K; k++) st[k] = win[k];
    }
    act[(size_t)b * conv_dim + c] = m2_silu(acc);
}

// LPR lanes per state row (S / 4 floats per lane group, float4 each), 32 / LPR rows per
// warp pass.  The CTA covers rows [r0, r0 + kM2Rows) of head h of sequence b.
template <int LPR>
__global__ void __launch_bounds__(kM2Threads) k_m2_scan(const float *__restrict__ act, const float *__restrict__ z,
                                                        int z_stride, const float *__restrict__ dt, int dt_stride,
                                                        const float *__restrict__ A_log,
                                                        const float *__restrict__ dt_bias,
                                                        const float *__restrict__ Dv, float *__restrict__ state,
                                                        float *__restrict__ y, int H, int P, int S, int G) {
    extern __shared__ float m2_sm[];                 // B [S], C [S]
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y;
    const int tiles = P / kM2Rows;
    const int h = blockIdx.x / tiles, r0 = (blockIdx.x % tiles) * kM2Rows;
    const int g = h / (H / G);
    const int d_inner = H * P, conv_dim = d_inner + 2 * G * S;
    const float *a = act + (size_t)b * conv_dim;
    float *Bs = m2_sm, *Cs = m2_sm + S;
    for (int n = threadIdx.x; n < S; n += blockDim.x) {
        Bs[n] = a[d_inner + g * S + n];
        Cs[n] = a[d_inner + G * S + g * S + n];
    }
    __syncthreads();
    const float dtv = fmaxf(m2_softplus(dt[(size_t)b * dt_stride + h] + dt_bias[h]), 0.0f);
    const float dA = __expf(-__expf(A_log[h]) * dtv);
    const float Dh = Dv ? Dv[h] : 0.0f;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int RPW = 32 / LPR;                    // rows per warp pass
    const int sub = lane / LPR, ln = lane % LPR;
    const int n_per = S / (4 * LPR);                 // float4 groups per lane
    float *srow0 = state + (((size_t)b * H + h) * P) * S;
    for (int rr = warp * RPW; rr < kM2Rows; rr += (kM2Threads / 32) * RPW) {
        const int p = r0 + rr + sub;
        const float xp = a[h * P + p];
        const float dx = dtv * xp;
        float4 *srow = reinterpret_cast<float4 *>(srow0 + (size_t)p * S);
        float part = 0.0f;
        for (int j = 0; j < n_per; j++) {
            const int q = ln + j * LPR;              // float4 index in the row
            float4 s4 = srow[q];
            const float4 b4 = reinterpret_cast<const float4 *>(Bs)[q];
            const float4 c4 = reinterpret_cast<const float4 *>(Cs)[q];
            s4.x = fmaf(s4.x, dA, dx * b4.x);
            s4.y = fmaf(s4.y, dA, dx * b4.y);
            s4.z = fmaf(s4.z, dA, dx * b4.z);
            s4.w = fmaf(s4.w, dA, dx * b4.w);
            srow[q] = s4;
            part = fmaf(s4.x, c4.x, part);
            part = fmaf(s4.y, c4.y, part);
            part = fmaf(s4.z, c4.z, part);
            part = fmaf(s4.w, c4.w, part);
        }
#pragma unroll
        for (int o = LPR / 2; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (ln == 0) {
            float yp = fmaf(Dh, xp, part);
            if (z) yp *= m2_silu(z[(size_t)b * z_stride + h * P + p]);
            y[(size_t)b * d_inner + h * P + p] = yp;
        }
    }
}

// y <- norm_w * y / sqrt(mean(y^2) + eps) over each group of gs elements
__global__ void __launch_bounds__(256) k_m2_norm(float *__restrict__ y, const float *__restrict__ norm_w, int d_inner,
                                                 int gs, float eps) {
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.y, grp = blockIdx.x;
    float *row = y + (size_t)b * d_inner + (size_t)grp * gs;
    const float *w = norm_w + (size_t)grp * gs;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < gs; i += blockDim.x) ss = fmaf(row[i], row[i], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    __shared__ float red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = rsqrtf(v / (float)gs + eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int i = threadIdx.x; i < gs; i += blockDim.x) row[i] = row[i] * inv * w[i];
}

template <typename Kern, typename... Args>
static cudaError_t m2_launch(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, args...);
}

struct Mamba2Dims {
    int B, H, P, S, G, K, norm_group;
    float eps;
};

static const char *mamba2_bad_dims(const Mamba2Dims &d) {
    if (d.B <= 0 || d.H <= 0 || d.P <= 0 || d.S <= 0 || d.G <= 0 || d.K <= 0) return "non-positive size";
    if (d.H % d.G) return "heads not a multiple of groups";
    if (d.P % kM2Rows) return "head_dim not a multiple of 32";
    if (!(d.S == 16 || d.S == 32 || d.S == 64 || (d.S % 128 == 0 && d.S <= 4096)))
        return "state size not 16, 32, 64 or a multiple of 128 (<= 4096)";
    if (d.K > kM2MaxConv) return "conv width above 8";
    if (d.norm_group < 0 || (d.norm_group > 0 && (d.H * d.P) % d.norm_group)) return "norm group does not divide d_inner";
    return nullptr;
}

// act: [B][conv_dim] scratch; y: [B][H*P]
static int launch_mamba2(const Mamba2Dims &d, const float *xbc, int xbc_stride, const float *z, int z_stride,
                         const float *dt, int dt_stride, float *conv_state, const float *conv_w,
                         const float *conv_b, const float *A_log, const float *dt_bias, const float *Dv,
                         const float *norm_w, float *ssm_state, float *y, float *act, cudaStream_t s) {
    const int d_inner = d.H * d.P, conv_dim = d_inner + 2 * d.G * d.S;
    if (!MLQ_CUDA(m2_launch(k_m2_conv, dim3((conv_dim + 255) / 256, d.B), dim3(256), 0, s, xbc, xbc_stride,
                            conv_state, conv_w, conv_b, act, conv_dim, d.K)))
        return MLQ_ERR_CUDA;
    count_launch();
    const size_t smem = sizeof(float) * 2 * (size_t)d.S;
    const dim3 grid(d.H * (d.P / kM2Rows), d.B);
    const int lpr = d.S >= 128 ? 32 : d.S / 4;      // lanes per state row
    cudaError_t e;
    switch (lpr) {
        case 32: e = m2_launch(k_m2_scan<32>, grid, dim3(kM2Threads), smem, s, (const float *)act, z, z_stride, dt,
                               dt_stride, A_log, dt_bias, Dv, ssm_state, y, d.H, d.P, d.S, d.G); break;
        case 16: e = m2_launch(k_m2_scan<16>, grid, dim3(kM2Threads), smem, s, (const float *)act, z, z_stride, dt,
                               dt_stride, A_log, dt_bias, Dv, ssm_state, y, d.H, d.P, d.S, d.G); break;
        case 8: e = m2_launch(k_m2_scan<8>, grid, dim3(kM2Threads), smem, s, (const float *)act, z, z_stride, dt,
                              dt_stride, A_log, dt_bias, Dv, ssm_state, y, d.H, d.P, d.S, d.G); break;
        default: e = m2_launch(k_m2_scan<4>, grid, dim3(kM2Threads), smem, s, (const float *)act, z, z_stride, dt,
                               dt_stride, A_log, dt_bias, Dv, ssm_state, y, d.H, d.P, d.S, d.G); break;
    }
    if (!MLQ_CUDA(e)) return MLQ_ERR_CUDA;
    count_launch();
    if (norm_w) {
        const int gs = d.norm_group > 0 ? d.norm_group : d_inner;
        if (!MLQ_CUDA(m2_launch(k_m2_norm, dim3(d_inner / gs, d.B), dim3(256), 0, s, y, norm_w, d_inner, gs, d.eps)))
            return MLQ_ERR_CUDA;
        count_launch();
    }
    return MLQ_OK;
}

}  // namespace mlq

using namespace mlq;

extern "C" {

int mlq_mamba2_step(const float *xbc, const float *z, const float *dt, float *conv_state, const float *conv_w,
                    const float *conv_b, const float *A_log, const float *dt_bias, const float *D,
                    const float *norm_w, float *ssm_state, float *y, int B, int H, int P, int S, int G, int d_conv,
                    float eps, int norm_group) {
    const Mamba2Dims d{B, H, P, S, G, d_conv, norm_group, eps};
    if (const char *why = mamba2_bad_dims(d)) {
        set_error(MLQ_ERR_ARG, "mlq_mamba2_step: %s", why);
        return MLQ_ERR_ARG;
    }
    if (!xbc || !dt || !conv_state || !conv_w || !A_log || !dt_bias || !ssm_state || !y) {
        set_error(MLQ_ERR_ARG, "mlq_mamba2_step: null pointer");
        return MLQ_ERR_ARG;
    }
    const int d_inner = H * P, conv_dim = d_inner + 2 * G * S;
    CallScope cs;
    const float *dx = (const float *)cs.in(xbc, sizeof(float) * (size_t)B * conv_dim);
    const float *dz = z ? (const float *)cs.in(z, sizeof(float) * (size_t)B * d_inner) : nullptr;
    const float *ddt = (const float *)cs.in(dt, sizeof(float) * (size_t)B * H);
    float *dcs = (float *)cs.inout(conv_state, sizeof(float) * (size_t)B * conv_dim * d_conv);
    const float *dw = (const float *)cs.weights(conv_w, sizeof(float) * (size_t)conv_dim * d_conv);
    const float *db = conv_b ? (const float *)cs.weights(conv_b, sizeof(float) * conv_dim) : nullptr;
    const float *da = (const float *)cs.weights(A_log, sizeof(float) * H);
    const float *dtb = (const float *)cs.weights(dt_bias, sizeof(float) * H);
    const float *dd = D ? (const float *)cs.weights(D, sizeof(float) * H) : nullptr;
    const float *dn = norm_w ? (const float *)cs.weights(norm_w, sizeof(float) * d_inner) : nullptr;
    float *dss = (float *)cs.inout(ssm_state, sizeof(float) * (size_t)B * H * P * S);
    float *dy = (float *)cs.out(y, sizeof(float) * (size_t)B * d_inner);
    float *act = (float *)cs.scratch(sizeof(float) * (size_t)B * conv_dim);
    if (cs.failed) return cs.finish();
    int rc = launch_mamba2(d, dx, conv_dim, dz, d_inner, ddt, H, dcs, dw, db, da, dtb, dd, dn, dss, dy, act,
                           stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

// The mixer of one token per sequence: proj = W_in u (rows z | xBC | dt), the step, then
// out = W_out y.  W_in [H*P + conv_dim + H][hidden] of type qt_in, W_out [hidden][H*P] of
// type qt_out (any type mlq_matmul takes; 0 = F32).
int mlq_mamba2_layer(const float *u, int B, int hidden, const void *W_in, int qt_in, const void *W_out, int qt_out,
                     float *conv_state, const float *conv_w, const float *conv_b, const float *A_log,
                     const float *dt_bias, const float *D, const float *norm_w, float *ssm_state, float *out, int H,
                     int P, int S, int G, int d_conv, float eps, int norm_group) {
    const Mamba2Dims d{B, H, P, S, G, d_conv, norm_group, eps};
    if (const char *why = mamba2_bad_dims(d)) {
        set_error(MLQ_ERR_ARG, "mlq_mamba2_layer: %s", why);
        return MLQ_ERR_ARG;
    }
    if (!u || !W_in || !W_out || !conv_state || !conv_w || !A_log || !dt_bias || !ssm_state || !out || hidden <= 0) {
        set_error(MLQ_ERR_ARG, "mlq_mamba2_layer: null pointer or hidden <= 0");
        return MLQ_ERR_ARG;
    }
    const int d_inner = H * P, conv_dim = d_inner + 2 * G * S, n_proj = d_inner + conv_dim + H;
    const size_t rb_in = mlq_row_bytes(qt_in, hidden), rb_out = mlq_row_bytes(qt_out, d_inner);
    if (!rb_in || !rb_out) {
        set_error(MLQ_ERR_TYPE, "mlq_mamba2_layer: weight type %d / %d with rows of %d / %d", qt_in, qt_out, hidden,
                  d_inner);
        return MLQ_ERR_TYPE;
    }
    CallScope cs;
    const float *du = (const float *)cs.in(u, sizeof(float) * (size_t)B * hidden);
    const uint8_t *wi = (const uint8_t *)cs.weights(W_in, rb_in * n_proj);
    const uint8_t *wo = (const uint8_t *)cs.weights(W_out, rb_out * hidden);
    float *dcs = (float *)cs.inout(conv_state, sizeof(float) * (size_t)B * conv_dim * d_conv);
    const float *dw = (const float *)cs.weights(conv_w, sizeof(float) * (size_t)conv_dim * d_conv);
    const float *db = conv_b ? (const float *)cs.weights(conv_b, sizeof(float) * conv_dim) : nullptr;
    const float *da = (const float *)cs.weights(A_log, sizeof(float) * H);
    const float *dtb = (const float *)cs.weights(dt_bias, sizeof(float) * H);
    const float *dd = D ? (const float *)cs.weights(D, sizeof(float) * H) : nullptr;
    const float *dn = norm_w ? (const float *)cs.weights(norm_w, sizeof(float) * d_inner) : nullptr;
    float *dss = (float *)cs.inout(ssm_state, sizeof(float) * (size_t)B * H * P * S);
    float *dout = (float *)cs.out(out, sizeof(float) * (size_t)B * hidden);
    float *proj = (float *)cs.scratch(sizeof(float) * (size_t)B * n_proj);
    float *act = (float *)cs.scratch(sizeof(float) * (size_t)B * conv_dim);
    float *y = (float *)cs.scratch(sizeof(float) * (size_t)B * d_inner);
    if (cs.failed) return cs.finish();
    cudaStream_t s = stream();
    int rc = launch_matmul(wi, qt_in, du, proj, n_proj, hidden, B, rb_in * n_proj, s);
    if (rc == MLQ_OK)
        rc = launch_mamba2(d, proj + d_inner, n_proj, proj, n_proj, proj + d_inner + conv_dim, n_proj, dcs, dw, db, da,
                           dtb, dd, dn, dss, y, act, s);
    if (rc == MLQ_OK) rc = launch_matmul(wo, qt_out, y, dout, hidden, d_inner, B, rb_out * hidden, s);
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

}  // extern "C"
