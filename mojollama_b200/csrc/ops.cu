// Elementwise / row-wise ops of the reference engine as device kernels:
//   RMSNorm   simd_ops.c:35 (eps arg), quant_kernels_omp.c:956 (eps 1e-5),
//             cengine_batch_instr.c:1258-1279 (RMS_NORM_SIMD: NaN->0, clamp +-1000,
//             residual copy)                                    -> mlq_rms_norm
//   SiLU      simd_ops.c:56 (Pade tanh on the 8-wide body, expf on the tail),
//             quant_kernels_omp.c:981/1017 (exact expf)          -> mlq_silu
//   SiLU*up   quant_kernels_omp.c:2157-2164 (clamp +-80, exact)  -> mlq_swiglu
//   residual  simd_ops.c:77                                      -> mlq_add
//   softmax   quant_kernels_omp.c:1000, simd_ops.c:88            -> mlq_softmax
//   RoPE      simd_ops.c:122 (interleaved pairs, powf freq),
//             cengine_batch_instr.c:674-712 (rope_init tables, NeoX half split)
// All are HBM/launch bound; in the fused forward they are folded into neighbours.
#include <cuda_runtime.h>
#include <math.h>
#include <stdlib.h>

#include "formats.cuh"
#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

__device__ __forceinline__ float block_sum(float v, float *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        v = (l < (int)(blockDim.x >> 5)) ? sh[l] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (l == 0) sh[0] = v;
    }
    __syncthreads();
    return sh[0];
}

__device__ __forceinline__ float block_max(float v, float *sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    if (w == 0) {
        v = (l < (int)(blockDim.x >> 5)) ? sh[l] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (l == 0) sh[0] = v;
    }
    __syncthreads();
    return sh[0];
}

// one CTA per row.  flags bit0: sanitize (NaN->0, clamp +-1000) and write the clamped
// input to `res` (the reference's residual copy); bit1: in-place allowed (always true)
__global__ void k_rms_norm(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ w,
                           float *__restrict__ res, int n, float eps, int flags) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    __shared__ float sh[32];
    const float *xr = x + (size_t)blockIdx.x * n;
    float *orow = out + (size_t)blockIdx.x * n;
    float ss = 0.0f;
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i];
        if (flags & 1) {
            if (v != v) v = 0.0f;
            v = fminf(fmaxf(v, -1000.0f), 1000.0f);
            if (res) res[(size_t)blockIdx.x * n + i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, sh);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i];
        if (flags & 1) {
            if (v != v) v = 0.0f;
            v = fminf(fmaxf(v, -1000.0f), 1000.0f);
        }
        orow[i] = (v * inv) * (w ? w[i] : 1.0f);
    }
}

// x += y on the row, then k_rms_norm of the new row (res null): one launch for the residual add
// of a block's output and the next block's norm.  Each thread re-reads only what it wrote.
__global__ void k_add_rms_norm(float *__restrict__ x, const float *__restrict__ y, const float *__restrict__ w,
                               float *__restrict__ out, int n, float eps, int flags) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    __shared__ float sh[32];
    float *xr = x + (size_t)blockIdx.x * n;
    const float *yr = y + (size_t)blockIdx.x * n;
    float *orow = out + (size_t)blockIdx.x * n;
    float ss = 0.0f;
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i] + yr[i];
        xr[i] = v;
        if (flags & 1) {
            if (v != v) v = 0.0f;
            v = fminf(fmaxf(v, -1000.0f), 1000.0f);
        }
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, sh);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i];
        if (flags & 1) {
            if (v != v) v = 0.0f;
            v = fminf(fmaxf(v, -1000.0f), 1000.0f);
        }
        orow[i] = (v * inv) * (w ? w[i] : 1.0f);
    }
}

// k_rms_norm with the normalised row also written as a packed activation row (the
// input encoding of the GEMVs that read it).  CTA (slice, row): every CTA of a row sums the
// squares of the whole row (one pass over n floats), then normalises and encodes only its
// slice of 32-element blocks, warp w taking blocks w, w + 8, ... of the slice -- several
// CTAs per row keep this latency-bound step short.
__global__ void __launch_bounds__(256) k_rms_norm_encode(float *__restrict__ out, const float *__restrict__ x,
                                                          const float *__restrict__ w, float *__restrict__ res, int n,
                                                          float eps, int flags, uint8_t *__restrict__ planes) {
    __shared__ float sh[32];
    pdl_wait();
    pdl_trigger();
    const int row = blockIdx.y;
    const float *xr = x + (size_t)row * n;
    float ss = 0.0f;
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = xr[i];
        if (flags & 1) {
            if (v != v) v = 0.0f;
            v = fminf(fmaxf(v, -1000.0f), 1000.0f);
        }
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, sh);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int nb = n / 32, per = (nb + gridDim.x - 1) / gridDim.x;
    const int kb0 = blockIdx.x * per, kb1 = min(nb, kb0 + per);
    for (int kb = kb0 + warp; kb < kb1; kb += nw) {
        const int i = 32 * kb + lane;
        float v = xr[i];
        if (flags & 1) {
            if (v != v) v = 0.0f;
            v = fminf(fmaxf(v, -1000.0f), 1000.0f);
            if (res) res[(size_t)row * n + i] = v;
        }
        const float o = (v * inv) * (w ? w[i] : 1.0f);
        if (out) out[(size_t)row * n + i] = o;
        encode_block_packed(o, row, kb, n, planes, lane);
    }
}

// mode 0: exact x/(1+exp(-x)); mode 1: simd_ops.c's Pade tanh body + exact tail
__global__ void k_silu(float *__restrict__ out, const float *__restrict__ x, long long n, int mode) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const long long body = (mode == 1) ? (n - n % 8) : 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        float r;
        if (i < body) {
            const float h = v * 0.5f;
            const float v2 = h * h;
            const float num = h * (27.0f + v2);
            const float den = 27.0f + 9.0f * v2;
            const float t = num / den;
            r = v * (0.5f + 0.5f * t);
        } else if (mode == 1) {
            r = v * (1.0f / (1.0f + expf(-v)));
        } else {
            r = v / (1.0f + expf(-v));
        }
        out[i] = r;
    }
}

// h = silu(clamp(g, -80, 80)) * u   (quant_kernels_omp.c:2157-2164)
__global__ void k_swiglu(float *__restrict__ h, const float *__restrict__ g, const float *__restrict__ u, long long n) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        float gv = fminf(fmaxf(g[i], -80.0f), 80.0f);
        h[i] = (gv / (1.0f + expf(-gv))) * u[i];
    }
}

__global__ void k_add(float *__restrict__ out, const float *__restrict__ a, const float *__restrict__ b, long long n) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = a[i] + b[i];
}

// in place, one CTA per row
__global__ void k_softmax(float *__restrict__ x, int n) {
    __shared__ float sh[32];
    float *xr = x + (size_t)blockIdx.x * n;
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, xr[i]);
    mx = block_max(mx, sh);
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(xr[i] - mx);
        xr[i] = e;
        s += e;
    }
    s = block_sum(s, sh);
    const float inv = 1.0f / s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xr[i] *= inv;
}

// simd_ops.c:122 apply_rope: pairs (d, d+1), freq = 1/powf(base, (d/2)/(hd/2))
__global__ void k_rope_interleaved(float *__restrict__ q, float *__restrict__ k, int nh, int nkh, int hd, int pos,
                                   float base) {
    const int pairs = hd / 2;
    const int total = (nh + nkh) * pairs;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int head = t / pairs, p = t - head * pairs, d = 2 * p;
        float *v = head < nh ? q + (size_t)head * hd : k + (size_t)(head - nh) * hd;
        const float freq = 1.0f / powf(base, (float)(d / 2) / (float)(hd / 2));
        const float ang = (float)pos * freq;
        const float c = cosf(ang), s = sinf(ang);
        const float a0 = v[d], a1 = v[d + 1];
        v[d] = a0 * c - a1 * s;
        v[d + 1] = a0 * s + a1 * c;
    }
}

// cengine_batch_instr.c:674 rope_init: theta = pos / 10000^(2j/hd) in double
__global__ void k_rope_init(float *cos_t, float *sin_t, int max_ctx, int hd, int rope_dim, double base) {
    const int hd2 = rope_dim / 2;
    const long long total = (long long)max_ctx * hd2;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {
        const int pos = (int)(t / hd2), j = (int)(t - (long long)pos * hd2);
        const double theta = (double)pos / pow(base, 2.0 * j / hd);
        cos_t[t] = (float)cos(theta);
        sin_t[t] = (float)sin(theta);
    }
}

// cengine_batch_instr.c:686 rope_apply: NeoX half split (j, j + rope_dim/2) of each head
__global__ void k_rope_neox(float *__restrict__ buf, int nh, int hd, const int *__restrict__ pos_dev, int pos_host,
                            const float *__restrict__ cos_t, const float *__restrict__ sin_t, int rope_dim,
                            int rows_stride) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const int hd2 = rope_dim / 2;
    const int row = blockIdx.y;
    const int pos = pos_dev ? pos_dev[row] : pos_host;
    float *b = buf + (size_t)row * rows_stride;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < nh * hd2; t += gridDim.x * blockDim.x) {
        const int h = t / hd2, j = t - h * hd2;
        float *v = b + (size_t)h * hd;
        const float c = cos_t[(size_t)pos * hd2 + j], s = sin_t[(size_t)pos * hd2 + j];
        const float a0 = v[j], a1 = v[j + hd2];
        v[j] = a0 * c - a1 * s;
        v[j + hd2] = a1 * c + a0 * s;
    }
}

static int grid_for(long long n, int threads = 256) {
    Ctx *c = ctx();
    long long g = (n + threads - 1) / threads;
    const long long cap = (long long)(c ? c->num_sms : 148) * 16;
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

int launch_rms_norm(float *out, const float *x, const float *w, float *res, int rows, int n, float eps, int flags,
                    cudaStream_t s) {
    return MLQ_CUDA(launch_pdl_k(k_rms_norm, dim3(rows), dim3(256), 0, s, out, x, w, res, n, eps, flags)) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_add_rms_norm(float *x, const float *y, const float *w, float *out, int rows, int n, float eps, int flags,
                        cudaStream_t s) {
    return MLQ_CUDA(launch_pdl_k(k_add_rms_norm, dim3(rows), dim3(256), 0, s, x, y, w, out, n, eps, flags)) ? MLQ_OK
                                                                                                           : MLQ_ERR_CUDA;
}

int launch_rms_norm_encode(float *out, const float *x, const float *w, float *res, int rows, int n, float eps,
                           int flags, uint8_t *planes, cudaStream_t s) {
    if (n % 32 || !planes) return MLQ_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    // one 32-element block per warp; a single CTA per row when normalising in place (the
    // other CTAs of the row would still be reading x)
    const int slices = out == x ? 1 : (n / 32 + 7) / 8;
    cfg.gridDim = dim3(slices, rows);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = getenv("MLQ_NO_PDL") ? 0 : 1;
    count_launch();
    return MLQ_CUDA(cudaLaunchKernelEx(&cfg, k_rms_norm_encode, out, x, w, res, n, eps, flags, planes)) ? MLQ_OK
                                                                                                        : MLQ_ERR_CUDA;
}

int launch_silu(float *out, const float *x, long long n, int mode, cudaStream_t s) {
    return MLQ_CUDA(launch_pdl_k(k_silu, dim3(grid_for(n)), dim3(256), 0, s, out, x, n, mode)) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_swiglu(float *h, const float *g, const float *u, long long n, cudaStream_t s) {
    return MLQ_CUDA(launch_pdl_k(k_swiglu, dim3(grid_for(n)), dim3(256), 0, s, h, g, u, n)) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_add(float *out, const float *a, const float *b, long long n, cudaStream_t s) {
    return MLQ_CUDA(launch_pdl_k(k_add, dim3(grid_for(n)), dim3(256), 0, s, out, a, b, n)) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_softmax(float *x, int rows, int n, cudaStream_t s) {
    k_softmax<<<rows, 256, 0, s>>>(x, n);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_rope_interleaved(float *q, float *k, int nh, int nkh, int hd, int pos, float base, cudaStream_t s) {
    k_rope_interleaved<<<grid_for((long long)(nh + nkh) * hd / 2), 256, 0, s>>>(q, k, nh, nkh, hd, pos, base);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_rope_init(float *cos_t, float *sin_t, int max_ctx, int hd, int rope_dim, double base, cudaStream_t s) {
    k_rope_init<<<grid_for((long long)max_ctx * (rope_dim / 2)), 256, 0, s>>>(cos_t, sin_t, max_ctx, hd, rope_dim, base);
    count_launch();
    return MLQ_CUDA(cudaGetLastError()) ? MLQ_OK : MLQ_ERR_CUDA;
}

int launch_rope_neox(float *buf, int rows, int rows_stride, int nh, int hd, const int *pos_dev, int pos_host,
                     const float *cos_t, const float *sin_t, int rope_dim, cudaStream_t s) {
    dim3 grid(grid_for((long long)nh * (rope_dim / 2)) > 64 ? 64 : grid_for((long long)nh * (rope_dim / 2)), rows);
    return MLQ_CUDA(launch_pdl_k(k_rope_neox, dim3(grid), dim3(256), 0, s, buf, nh, hd, pos_dev, pos_host, cos_t, sin_t, rope_dim, rows_stride)) ? MLQ_OK : MLQ_ERR_CUDA;
}

}  // namespace mlq

// ====================================================================================== C-ABI
using namespace mlq;

namespace {
// in-place when out == x (host or device); otherwise separate in/out views
struct InOut {
    const float *in;
    float *out;
};
InOut in_out(CallScope &cs, const float *x, float *out, size_t bytes) {
    if ((const void *)x == (const void *)out) {
        float *d = (float *)cs.inout(out, bytes);
        return {d, d};
    }
    return {(const float *)cs.in(x, bytes), (float *)cs.out(out, bytes)};
}
int done(CallScope &cs, int rc) {
    if (rc != MLQ_OK) cs.failed = true;
    int f = cs.finish();
    return rc != MLQ_OK ? rc : f;
}
}  // namespace

extern "C" {

int mlq_rms_norm(float *out, const float *x, const float *w, int rows, int n, float eps, int sanitize, float *res) {
    if (!out || !x || rows <= 0 || n <= 0) { set_error(MLQ_ERR_ARG, "mlq_rms_norm: bad arguments"); return MLQ_ERR_ARG; }
    CallScope cs;
    const size_t bytes = sizeof(float) * (size_t)rows * n;
    InOut io = in_out(cs, x, out, bytes);
    const float *dw = w ? (const float *)cs.weights(w, sizeof(float) * (size_t)n) : nullptr;
    float *dres = res ? (float *)cs.out(res, bytes) : nullptr;
    if (cs.failed) return cs.finish();
    return done(cs, launch_rms_norm(io.out, io.in, dw, dres, rows, n, eps, sanitize ? 1 : 0, stream()));
}

int mlq_silu(float *out, const float *x, long long n, int mode) {
    if (!out || !x || n <= 0) { set_error(MLQ_ERR_ARG, "mlq_silu: bad arguments"); return MLQ_ERR_ARG; }
    CallScope cs;
    InOut io = in_out(cs, x, out, sizeof(float) * (size_t)n);
    if (cs.failed) return cs.finish();
    return done(cs, launch_silu(io.out, io.in, n, mode, stream()));
}

int mlq_swiglu(float *h, const float *gate, const float *up, long long n) {
    if (!h || !gate || !up || n <= 0) { set_error(MLQ_ERR_ARG, "mlq_swiglu: bad arguments"); return MLQ_ERR_ARG; }
    CallScope cs;
    const size_t bytes = sizeof(float) * (size_t)n;
    const float *dg = (const float *)cs.in(gate, bytes);
    const float *du = (const float *)cs.in(up, bytes);
    float *dh = (float *)cs.out(h, bytes);
    if (cs.failed) return cs.finish();
    return done(cs, launch_swiglu(dh, dg, du, n, stream()));
}

int mlq_add(float *out, const float *a, const float *b, long long n) {
    if (!out || !a || !b || n <= 0) { set_error(MLQ_ERR_ARG, "mlq_add: bad arguments"); return MLQ_ERR_ARG; }
    CallScope cs;
    const size_t bytes = sizeof(float) * (size_t)n;
    const float *da, *db;
    float *dout;
    if (out == a || out == b) {
        dout = (float *)cs.inout(out, bytes);
        da = (out == a) ? dout : (const float *)cs.in(a, bytes);
        db = (out == b) ? dout : (const float *)cs.in(b, bytes);
    } else {
        da = (const float *)cs.in(a, bytes);
        db = (const float *)cs.in(b, bytes);
        dout = (float *)cs.out(out, bytes);
    }
    if (cs.failed) return cs.finish();
    return done(cs, launch_add(dout, da, db, n, stream()));
}

int mlq_softmax(float *x, int rows, int n) {
    if (!x || rows <= 0 || n <= 0) { set_error(MLQ_ERR_ARG, "mlq_softmax: bad arguments"); return MLQ_ERR_ARG; }
    CallScope cs;
    float *dx = (float *)cs.inout(x, sizeof(float) * (size_t)rows * n);
    if (cs.failed) return cs.finish();
    return done(cs, launch_softmax(dx, rows, n, stream()));
}

int mlq_rope_interleaved(float *q, float *k, int n_heads, int n_kv_heads, int head_dim, int pos, float base) {
    if (!q || !k || n_heads <= 0 || n_kv_heads < 0 || head_dim <= 0 || head_dim % 2) {
        set_error(MLQ_ERR_ARG, "mlq_rope_interleaved: bad arguments");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    float *dq = (float *)cs.inout(q, sizeof(float) * (size_t)n_heads * head_dim);
    float *dk = (float *)cs.inout(k, sizeof(float) * (size_t)(n_kv_heads > 0 ? n_kv_heads : 1) * head_dim);
    if (cs.failed) return cs.finish();
    return done(cs, launch_rope_interleaved(dq, dk, n_heads, n_kv_heads, head_dim, pos, base, stream()));
}

int mlq_rope_init(float *cos_t, float *sin_t, int max_ctx, int head_dim, int rope_dim, double base) {
    if (rope_dim <= 0) rope_dim = head_dim;
    if (!cos_t || !sin_t || max_ctx <= 0 || head_dim <= 0 || rope_dim > head_dim) {
        set_error(MLQ_ERR_ARG, "mlq_rope_init: bad arguments");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    const size_t bytes = sizeof(float) * (size_t)max_ctx * (rope_dim / 2);
    float *dc = (float *)cs.out(cos_t, bytes);
    float *ds = (float *)cs.out(sin_t, bytes);
    if (cs.failed) return cs.finish();
    return done(cs, launch_rope_init(dc, ds, max_ctx, head_dim, rope_dim, base, stream()));
}

int mlq_rope_neox(float *buf, int rows, int row_stride, int n_heads, int head_dim, const int *pos, int pos_scalar,
                  const float *cos_t, const float *sin_t, int rope_dim, int max_ctx) {
    if (rope_dim <= 0) rope_dim = head_dim;
    if (!buf || !cos_t || !sin_t || rows <= 0 || n_heads <= 0 || rope_dim > head_dim || max_ctx <= 0) {
        set_error(MLQ_ERR_ARG, "mlq_rope_neox: bad arguments");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    if (row_stride <= 0) row_stride = n_heads * head_dim;
    float *db = (float *)cs.inout(buf, sizeof(float) * (size_t)((rows - 1) * (size_t)row_stride + n_heads * head_dim));
    const int *dp = pos ? (const int *)cs.in(pos, sizeof(int) * (size_t)rows) : nullptr;
    const size_t tb = sizeof(float) * (size_t)max_ctx * (rope_dim / 2);
    const float *dc = (const float *)cs.weights(cos_t, tb);
    const float *dsn = (const float *)cs.weights(sin_t, tb);
    if (cs.failed) return cs.finish();
    return done(cs, launch_rope_neox(db, rows, row_stride, n_heads, head_dim, dp, pos_scalar, dc, dsn, rope_dim, stream()));
}

}  // extern "C"
