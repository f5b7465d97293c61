// SSM decode step of the reference engine (cengine_batch_instr.c:736-797) and the
// fused SSM layer around it (cengine_batch_instr.c:803-849), as device kernels.
//
// ssm_decode_step computes, for each sequence b (one token each):
//   conv[i]  = x_b[i % N] * conv1d_w[i]                 i < 2*inner (first conv tap only)
//   interm_b = silu(conv[0:inner]) * conv[inner:2*inner]
// and updates the state shared by all sequences, group by group, in sequence order:
//   dt  = softplus(dt_bias[g] + sum_j alpha[g][j] * x_b[j % N])   (softplus = x above 20)
//   state[g][s] = exp(a[g] * dt) * state[g][s] + (s == 0 ? dt * sum_j beta[g][j] * x_b[j % N] : 0)
// The state never feeds the output.  These are the reference's semantics, kept for the
// drop-in (only the first conv tap is used, the state is shared by the batch and is never
// read back, so this is not a Mamba-2 step); one launch computes
// the gated intermediate, one the state update (a thread per (group, state) element
// walking the B updates in order, so the result is deterministic).
// ssm_layer_fused: out_b = residual_b + W_out . ((W_gate . x_b) * interm_b).
#include <cuda_runtime.h>
#include <math.h>

#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

__global__ void k_ssm_interm(const float *__restrict__ x, const float *__restrict__ conv_w, float *__restrict__ interm,
                             int B, int N, int inner) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    const long long total = (long long)B * inner;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(t / inner), i = (int)(t - (long long)b * inner);
        const float *xb = x + (size_t)b * N;
        const float g = xb[i % N] * conv_w[i];
        const float v = xb[(i + inner) % N] * conv_w[i + inner];
        interm[t] = (g / (1.0f + expf(-g))) * v;
    }
}

// one block per group: dt and the B-term per sequence, then the ordered state update
__global__ void k_ssm_state(const float *__restrict__ x, const float *__restrict__ a_param,
                            const float *__restrict__ dt_bias, const float *__restrict__ alpha,
                            const float *__restrict__ beta, float *__restrict__ state, int B, int N, int state_size,
                            int dt_rank) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    extern __shared__ float sh[];   // [B] a_disc, [B] bx
    const int g = blockIdx.x;
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        const float *xb = x + (size_t)b * N;
        float dt = dt_bias[g];
        float bx = 0.0f;
        for (int j = 0; j < dt_rank; j++) {
            dt += alpha[(size_t)g * dt_rank + j] * xb[j % N];
            bx += beta[(size_t)g * dt_rank + j] * xb[j % N];
        }
        dt = dt > 20.0f ? dt : logf(1.0f + expf(dt));
        sh[b] = expf(a_param[g] * dt);
        sh[B + b] = bx * dt;
    }
    __syncthreads();
    float *sg = state + (size_t)g * state_size;
    for (int s = threadIdx.x; s < state_size; s += blockDim.x) {
        float v = sg[s];
        for (int b = 0; b < B; b++) v = sh[b] * v + (s == 0 ? sh[B + b] : 0.0f);
        sg[s] = v;
    }
}

__global__ void k_mul(float *__restrict__ a, const float *__restrict__ b, long long n) {
    pdl_wait();   // programmatic dependent launch: nothing is touched before the previous kernel ends
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        a[i] *= b[i];
}

int launch_ssm_decode_step(const float *x, float *interm, const float *conv_w, const float *a_param,
                           const float *dt_bias, const float *alpha, const float *beta, float *state, int B, int N,
                           int inner, int groups, int state_size, int dt_rank, cudaStream_t s) {
    const long long total = (long long)B * inner;
    int grid = (int)((total + 255) / 256);
    if (grid > 4096) grid = 4096;
    if (!MLQ_CUDA(launch_pdl_k(k_ssm_interm, dim3(grid), dim3(256), 0, s, x, conv_w, interm, B, N, inner)))
        return MLQ_ERR_CUDA;
    return MLQ_CUDA(launch_pdl_k(k_ssm_state, dim3(groups), dim3(128), sizeof(float) * 2 * B, s, x, a_param, dt_bias,
                                 alpha, beta, state, B, N, state_size, dt_rank))
               ? MLQ_OK
               : MLQ_ERR_CUDA;
}

int launch_mul(float *a, const float *b, long long n, cudaStream_t s) {
    int grid = (int)((n + 255) / 256);
    if (grid > 4096) grid = 4096;
    return MLQ_CUDA(launch_pdl_k(k_mul, dim3(grid), dim3(256), 0, s, a, b, n)) ? MLQ_OK : MLQ_ERR_CUDA;
}

}  // namespace mlq

// ====================================================================================== C-ABI
using namespace mlq;

extern "C" {

int mlq_ssm_decode_step(const float *x, float *interm, const float *conv1d_w, const float *a_param,
                        const float *dt_bias, const float *alpha, const float *beta, const float *ssm_norm_w,
                        float *state, int B, int N, int inner, int groups, int state_size, int conv_kernel,
                        int dt_rank) {
    (void)ssm_norm_w;
    (void)conv_kernel;
    if (!x || !interm || !conv1d_w || !a_param || !dt_bias || !alpha || !beta || !state || B <= 0 || N <= 0 ||
        inner <= 0 || groups <= 0 || state_size <= 0 || dt_rank < 0) {
        set_error(MLQ_ERR_ARG, "ssm_decode_step: bad arguments");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    const float *dx = (const float *)cs.in(x, sizeof(float) * (size_t)B * N);
    const float *dc = (const float *)cs.weights(conv1d_w, sizeof(float) * (size_t)2 * inner);
    const float *da = (const float *)cs.weights(a_param, sizeof(float) * (size_t)groups);
    const float *db = (const float *)cs.weights(dt_bias, sizeof(float) * (size_t)groups);
    const float *dal = (const float *)cs.weights(alpha, sizeof(float) * (size_t)groups * (dt_rank > 0 ? dt_rank : 1));
    const float *dbe = (const float *)cs.weights(beta, sizeof(float) * (size_t)groups * (dt_rank > 0 ? dt_rank : 1));
    float *dst = (float *)cs.inout(state, sizeof(float) * (size_t)groups * state_size);
    float *dint = (float *)cs.out(interm, sizeof(float) * (size_t)B * inner);
    if (cs.failed) return cs.finish();
    int rc = launch_ssm_decode_step(dx, dint, dc, da, db, dal, dbe, dst, B, N, inner, groups, state_size, dt_rank,
                                    stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

int mlq_ssm_layer_fused(const float *x, const float *residual, float *output, const float *conv1d_w,
                        const float *a_param, const float *dt_bias, const float *alpha, const float *beta,
                        const float *ssm_norm_w, float *state, const void *gate_raw, int gate_nr, int gate_nc,
                        int gate_qt, const void *ssm_out_raw, int ssm_out_nr, int ssm_out_nc, int ssm_out_qt, int B,
                        int N, int inner, int groups, int state_size, int conv_kernel, int dt_rank) {
    (void)ssm_norm_w;
    (void)conv_kernel;
    if (!x || !residual || !output || !gate_raw || !ssm_out_raw || B <= 0 || gate_nr != inner || gate_nc != N ||
        ssm_out_nr != N || ssm_out_nc != inner) {
        set_error(MLQ_ERR_ARG, "ssm_layer_fused: bad arguments (gate %dx%d, out %dx%d, N %d, inner %d)", gate_nr,
                  gate_nc, ssm_out_nr, ssm_out_nc, N, inner);
        return MLQ_ERR_ARG;
    }
    const size_t rbg = mlq_row_bytes(gate_qt, gate_nc), rbo = mlq_row_bytes(ssm_out_qt, ssm_out_nc);
    if (!rbg || !rbo) { set_error(MLQ_ERR_TYPE, "ssm_layer_fused: types %d/%d", gate_qt, ssm_out_qt); return MLQ_ERR_TYPE; }
    CallScope cs;
    const float *dx = (const float *)cs.in(x, sizeof(float) * (size_t)B * N);
    const float *dr = (const float *)cs.in(residual, sizeof(float) * (size_t)B * N);
    const float *dc = (const float *)cs.weights(conv1d_w, sizeof(float) * (size_t)2 * inner);
    const float *da = (const float *)cs.weights(a_param, sizeof(float) * (size_t)groups);
    const float *db = (const float *)cs.weights(dt_bias, sizeof(float) * (size_t)groups);
    const float *dal = (const float *)cs.weights(alpha, sizeof(float) * (size_t)groups * (dt_rank > 0 ? dt_rank : 1));
    const float *dbe = (const float *)cs.weights(beta, sizeof(float) * (size_t)groups * (dt_rank > 0 ? dt_rank : 1));
    float *dst = (float *)cs.inout(state, sizeof(float) * (size_t)groups * state_size);
    const uint8_t *dg = (const uint8_t *)cs.weights(gate_raw, rbg * gate_nr);
    const uint8_t *dout_w = (const uint8_t *)cs.weights(ssm_out_raw, rbo * ssm_out_nr);
    float *interm = (float *)cs.scratch(sizeof(float) * (size_t)B * inner);
    float *gbuf = (float *)cs.scratch(sizeof(float) * (size_t)B * inner);
    float *oproj = (float *)cs.scratch(sizeof(float) * (size_t)B * N);
    float *dout = (float *)cs.out(output, sizeof(float) * (size_t)B * N);
    if (cs.failed) return cs.finish();
    cudaStream_t s = stream();
    int rc = launch_ssm_decode_step(dx, interm, dc, da, db, dal, dbe, dst, B, N, inner, groups, state_size, dt_rank, s);
    if (rc == MLQ_OK) rc = launch_matmul(dg, gate_qt, dx, gbuf, inner, N, B, rbg * inner, s);
    if (rc == MLQ_OK) rc = launch_mul(interm, gbuf, (long long)B * inner, s);
    if (rc == MLQ_OK) rc = launch_matmul(dout_w, ssm_out_qt, interm, oproj, N, inner, B, rbo * N, s);
    if (rc == MLQ_OK) rc = launch_add(dout, dr, oproj, (long long)B * N, s);
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

}  // extern "C"
