// Plain GEMMs of 16-bit float weight matrices (bf16 / f16 tensors of a GGUF file: the
// GPT-OSS attention projections and output head) with more than a few activation rows.
//
// The reference has no GPU path for these: quant_matmul_omp has no F16/BF16 case
// (quant_kernels_omp.c:1355-1388) and its Python dequantizes them to F32 for numpy
// (turbo_engine_v7_moe.py:456-489).  With 1-4 activation rows the library's own GEMV reads
// the matrix once; with more it would re-read it in passes of four rows, so these go to a
// cuBLAS GEMM (a plain library GEMM: the weights as stored, fp32 accumulation).  The fp32
// activations enter as two 16-bit parts, x = hi + lo with hi = rn(x) and lo = rn(x - hi),
// accumulated into the same fp32 output (beta = 1 for the second product): ~16 mantissa
// bits of each activation, relative error ~1e-5, inside the 1e-3 bar of a single matmul.
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <type_traits>

#include "mlq_internal.h"
#include "pipeline.cuh"

namespace mlq {

template <typename T>
__global__ void k_split16(const float *__restrict__ x, T *__restrict__ hi, T *__restrict__ lo, long long n) {
    pdl_wait();
    pdl_trigger();
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        T h, l;
        if constexpr (sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value) {
            h = __float2bfloat16_rn(v);
            l = __float2bfloat16_rn(v - __bfloat162float(h));
        } else {
            h = __float2half_rn(v);
            l = __float2half_rn(v - __half2float(h));
        }
        hi[i] = h;
        lo[i] = l;
    }
}

struct BlasHandle {
    cublasHandle_t h = nullptr;
    void *ws = nullptr;
};
static std::mutex g_blas_mu;
static std::map<int, BlasHandle> g_blas;
static constexpr size_t kBlasWorkspace = (size_t)32 << 20;

// the device's handle with its own workspace (so that a captured stream never makes cuBLAS
// allocate), created outside any capture; null when cuBLAS is unavailable
static cublasHandle_t blas_handle(cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_blas_mu);
    BlasHandle &b = g_blas[dev];
    if (!b.h) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
            cudaGetLastError();
            return nullptr;
        }
        if (cublasCreate(&b.h) != CUBLAS_STATUS_SUCCESS) { b.h = nullptr; return nullptr; }
        if (cudaMalloc(&b.ws, kBlasWorkspace) != cudaSuccess ||
            cublasSetWorkspace(b.h, b.ws, kBlasWorkspace) != CUBLAS_STATUS_SUCCESS) {
            cudaGetLastError();
            cublasDestroy(b.h);
            b.h = nullptr;
            return nullptr;
        }
        cublasSetMathMode(b.h, CUBLAS_DEFAULT_MATH);
    }
    if (cublasSetStream(b.h, s) != CUBLAS_STATUS_SUCCESS) return nullptr;
    return b.h;
}

// out[B][N] = x[B][K] . W[N][K]^T for 16-bit W (bf16: wt16 = 1, f16: 0); MLQ_ERR_UNSUPPORTED
// when cuBLAS or the scratch is not available (the caller then uses its GEMV passes)
int launch_gemm16(const void *W, int bf16, const float *x, float *out, int n_rows, int K, int B, cudaStream_t s) {
    const LaunchEnv *env = launch_env();
    if (!env || env->no_alloc || K % 8 || (reinterpret_cast<uintptr_t>(W) & 15)) return MLQ_ERR_UNSUPPORTED;
    cublasHandle_t h = blas_handle(s);
    if (!h) return MLQ_ERR_UNSUPPORTED;
    const size_t n = (size_t)B * K;
    uint8_t *scr = static_cast<uint8_t *>(tc_scratch(s, 2 * n * 2 + 256));
    if (!scr) return MLQ_ERR_UNSUPPORTED;
    void *hi = scr, *lo = scr + ((n * 2 + 255) & ~(size_t)255);
    const unsigned grid = (unsigned)((n + 255) / 256 > 2048 ? 2048 : (n + 255) / 256);
    if (bf16) k_split16<__nv_bfloat16><<<grid, 256, 0, s>>>(x, (__nv_bfloat16 *)hi, (__nv_bfloat16 *)lo, (long long)n);
    else k_split16<__half><<<grid, 256, 0, s>>>(x, (__half *)hi, (__half *)lo, (long long)n);
    count_launch();
    if (!MLQ_CUDA(cudaGetLastError())) return MLQ_ERR_CUDA;
    const cudaDataType_t t = bf16 ? CUDA_R_16BF : CUDA_R_16F;
    const float one = 1.0f, zero = 0.0f;
    // column-major view: C (N x B, ldc N) = W^T-as-stored (K x N, lda K)^T . X (K x B, ldb K)
    cublasStatus_t st = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, n_rows, B, K, &one, W, t,
                                     K, hi, t, K, &zero, out, CUDA_R_32F, n_rows, CUBLAS_COMPUTE_32F,
                                     CUBLAS_GEMM_DEFAULT);
    if (st == CUBLAS_STATUS_SUCCESS)
        st = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, n_rows, B, K, &one, W, t, K, lo, t, K, &one, out, CUDA_R_32F,
                          n_rows, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
    count_launch(2);
    if (st != CUBLAS_STATUS_SUCCESS) {
        set_error(MLQ_ERR_CUDA, "cublasGemmEx failed (%d)", (int)st);
        return MLQ_ERR_CUDA;
    }
    return MLQ_OK;
}

}  // namespace mlq
