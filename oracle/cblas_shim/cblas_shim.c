/* Naive SGEMM used only to let the reference's gqa_attention.c compile for the
 * oracle (see cblas.h in this folder).  C = alpha * op(A) * op(B) + beta * C.
 * Accumulates each dot product in double and rounds once, so its rounding is
 * at least as good as OpenBLAS's fp32 kernels. */
#include "cblas.h"

void openblas_set_num_threads(int n) { (void)n; }

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float *a, int lda,
                 const float *b, int ldb, float beta, float *c, int ldc) {
    if (order == CblasColMajor) {
        /* (C^T) = op(B)^T op(A)^T in row-major terms */
        cblas_sgemm(CblasRowMajor, tb, ta, n, m, k, alpha, b, ldb, a, lda, beta, c, ldc);
        return;
    }
    for (int i = 0; i < m; i++) {
        for (int j = 0; j < n; j++) {
            double acc = 0.0;
            for (int p = 0; p < k; p++) {
                float av = (ta == CblasNoTrans) ? a[(long)i * lda + p] : a[(long)p * lda + i];
                float bv = (tb == CblasNoTrans) ? b[(long)p * ldb + j] : b[(long)j * ldb + p];
                acc += (double)av * (double)bv;
            }
            float prev = (beta == 0.0f) ? 0.0f : beta * c[(long)i * ldc + j];
            c[(long)i * ldc + j] = (float)(alpha * acc) + prev;
        }
    }
}
