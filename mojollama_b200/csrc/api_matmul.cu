// C-ABI: quantized matmul / dequantize / Q8_0 quantize (host- or device-pointer).
#include <cuda_runtime.h>

#include "mlq_internal.h"

using namespace mlq;

extern "C" {

int mlq_block_elems(int qt) { return block_elems(qt); }
int mlq_block_bytes(int qt) { return block_bytes(qt); }

size_t mlq_row_bytes(int qt, int n_cols) {
    const int be = block_elems(qt);
    if (be <= 0 || n_cols <= 0 || n_cols % be) return 0;
    return (size_t)(n_cols / be) * block_bytes(qt);
}

int mlq_matmul(const void *W, int qt, const float *x, float *out, int n_rows, int n_cols, int B) {
    if (!W || !x || !out || n_rows <= 0 || n_cols <= 0 || B <= 0) {
        set_error(MLQ_ERR_ARG, "mlq_matmul: null pointer or non-positive size (N=%d K=%d B=%d)", n_rows,
                  n_cols, B);
        return MLQ_ERR_ARG;
    }
    if (block_elems(qt) <= 0) {
        set_error(MLQ_ERR_TYPE, "mlq_matmul: unsupported quant type %d", qt);
        return MLQ_ERR_TYPE;
    }
    const size_t rb = mlq_row_bytes(qt, n_cols);
    if (!rb) {
        set_error(MLQ_ERR_ARG, "mlq_matmul: K=%d is not a multiple of the %d-element block of type %d", n_cols,
                  block_elems(qt), qt);
        return MLQ_ERR_ARG;
    }
    if (ref_compat() && qt == MLQ_MXFP4) qt = MLQ_MXFP4_REF;
    CallScope cs;
    const size_t wb = rb * (size_t)n_rows;
    const uint8_t *dW = (const uint8_t *)cs.weights(W, wb);
    const float *dx = (const float *)cs.in(x, sizeof(float) * (size_t)B * n_cols);
    // one activation row of a quantized matrix: the GEMV kernels store each output once
    // (the many-row kernels in one contiguous run per tile), so a pinned host `out` is
    // written in place instead of through a staging buffer and a copy after the kernel
    bool host_mapped = false;
    float *dout = (float *)(B == 1 && is_quant_type(qt) ? cs.out_direct(out, sizeof(float) * (size_t)n_rows, &host_mapped)
                                                        : cs.out(out, sizeof(float) * (size_t)B * n_rows));
    if (cs.failed) return cs.finish();
    int rc;
    if (host_mapped && launch_env()) {
        LaunchEnv env = *launch_env();
        env.out_host = true;
        LaunchEnvScope scope(&env);
        rc = launch_matmul(dW, qt, dx, dout, n_rows, n_cols, B, wb, stream());
    } else {
        rc = launch_matmul(dW, qt, dx, dout, n_rows, n_cols, B, wb, stream());
    }
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

int mlq_gemv_fused(int qt, int n, const void *const *W, const int *n_rows, float *const *out,
                   const float *const *res, int mode, const float *x, int B, int K) {
    if (n < 1 || n > 4 || !W || !n_rows || !out || !x || B < 1 || B > 8 || K <= 0 || mode < 0 || mode > 2 ||
        (mode == 1 && !res) || (mode == 2 && n != 2)) {
        set_error(MLQ_ERR_ARG, "mlq_gemv_fused: bad arguments (n 1..4, B 1..8, mode 0..2)");
        return MLQ_ERR_ARG;
    }
    if (!is_device_ptr(x)) {
        set_error(MLQ_ERR_ARG, "mlq_gemv_fused: device pointers only");
        return MLQ_ERR_ARG;
    }
    CallScope cs;
    uint8_t *planes = (uint8_t *)cs.scratch(packed_rows_bytes(B, K));
    if (cs.failed) return cs.finish();
    cudaStream_t s = stream();
    int rc = K % 32 ? MLQ_ERR_UNSUPPORTED : launch_encode_packed(x, nullptr, nullptr, B, K, planes, s);
    if (rc == MLQ_OK)
        rc = launch_gemv_seg(qt, n, (const uint8_t *const *)W, n_rows, out, mode == 1 ? res : nullptr, mode == 2,
                             planes, B, K, s);
    if (rc == MLQ_ERR_UNSUPPORTED) {
        set_error(rc, "mlq_gemv_fused: type %d, K=%d, B=%d not covered", qt, K, B);
        cs.finish();
        return rc;
    }
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

int mlq_dequantize(const void *W, int qt, float *out, int64_t n) {
    if (!W || !out || n <= 0) {
        set_error(MLQ_ERR_ARG, "mlq_dequantize: null pointer or non-positive n");
        return MLQ_ERR_ARG;
    }
    const int be = block_elems(qt);
    if (be <= 0) { set_error(MLQ_ERR_TYPE, "mlq_dequantize: unsupported type %d", qt); return MLQ_ERR_TYPE; }
    if (n % be) { set_error(MLQ_ERR_ARG, "mlq_dequantize: n=%lld not a multiple of %d", (long long)n, be); return MLQ_ERR_ARG; }
    CallScope cs;
    const uint8_t *dW = (const uint8_t *)cs.in(W, (size_t)(n / be) * block_bytes(qt));
    float *dout = (float *)cs.out(out, sizeof(float) * (size_t)n);
    if (cs.failed) return cs.finish();
    int rc = launch_dequantize(dW, qt, dout, n, stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

int mlq_quantize_q8_0(const float *x, uint8_t *q8, int64_t n) {
    if (!x || !q8 || n <= 0) { set_error(MLQ_ERR_ARG, "mlq_quantize_q8_0: null pointer or n<=0"); return MLQ_ERR_ARG; }
    CallScope cs;
    const int64_t nb = n / 32;
    const float *dx = (const float *)cs.in(x, sizeof(float) * (size_t)(nb * 32));
    uint8_t *dq = (uint8_t *)cs.out(q8, (size_t)nb * 34);
    if (cs.failed) return cs.finish();
    if (nb > 0) {
        int rc = launch_quantize_q8_0(dx, dq, nb * 32, stream());
        if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    }
    return cs.finish();
}

int mlq_matmul_q8act(const void *W, int qt, const uint8_t *x_q8, float *out, int n_rows, int n_cols, int B) {
    if (!W || !x_q8 || !out || n_rows <= 0 || n_cols <= 0 || B <= 0 || n_cols % 32) {
        set_error(MLQ_ERR_ARG, "mlq_matmul_q8act: bad arguments");
        return MLQ_ERR_ARG;
    }
    const size_t rb = mlq_row_bytes(qt, n_cols);
    if (!rb) { set_error(MLQ_ERR_TYPE, "mlq_matmul_q8act: type %d / K=%d", qt, n_cols); return MLQ_ERR_TYPE; }
    if (ref_compat() && qt == MLQ_MXFP4) qt = MLQ_MXFP4_REF;
    CallScope cs;
    const uint8_t *dW = (const uint8_t *)cs.weights(W, rb * (size_t)n_rows);
    const uint8_t *dq = (const uint8_t *)cs.in(x_q8, (size_t)B * (n_cols / 32) * 34);
    float *dx = (float *)cs.scratch(sizeof(float) * (size_t)B * n_cols);
    float *dout = (float *)cs.out(out, sizeof(float) * (size_t)B * n_rows);
    if (cs.failed) return cs.finish();
    int rc = launch_q8act_to_f32(dq, dx, (int64_t)B * n_cols, stream());
    if (rc == MLQ_OK) rc = launch_matmul(dW, qt, dx, dout, n_rows, n_cols, B, rb * n_rows, stream());
    if (rc != MLQ_OK) { cs.failed = true; cs.finish(); return rc; }
    return cs.finish();
}

}  // extern "C"
